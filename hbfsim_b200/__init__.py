"""B200-native batched HBF access-timing path (HBFSim hot path).

The CUDA library libhbfsim_b200.so (hbfsim_b200/csrc) holds the kernels and
the C ABI; this package is the Python host side.  Importing it does not load
the library; `Context` does, and fails loudly if it is missing.
"""
from .api import (BatchResult, Context, HbfsimError, link_batch, link_profiles,  # noqa: F401
                  prefetch_sweep, submit_linked)
from ._lib import (ACCESS_BYPASS, ACCESS_FOREIGN, ACCESS_MODELED,  # noqa: F401
                   ACCESS_UNSUPPORTED, MODEL_DIE, MODEL_FAST, MODEL_HYBRID,
                   MODEL_REFERENCE, RANGE_CAPACITY, RANGE_TIMING)
