"""GPU parity of the UCIe streaming-link batch (reference:
hbfsim::ucie::StreamingLink, src/ucie/link.cpp, one thread per link):
delivery ticks, byte / flit counters, credits and the final tick equal to the
reference link's under the batch driver (tests/golden/link_goldens.json,
produced by the reference compiled from source) and to the oracle's
(oracle/hbf_oracle.c or_link_run, pinned to the same goldens)."""
import json
from pathlib import Path

import numpy as np
import pytest

import hbf_oracle as ho
from hbfsim_b200 import HbfsimError, link_batch, link_profiles

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "link_goldens.json"


def as_profiles(cases):
    ps = [c["profile"] for c in cases]
    return link_profiles(len(ps), [p["gt"] for p in ps], [p["ar"] for p in ps],
                         [p["r"] for p in ps], [p["accepted"] for p in ps],
                         [p["prop"] for p in ps], [p["consume"] for p in ps])


def run(cases):
    import torch
    offsets = np.cumsum([0] + [len(c["ready"]) for c in cases])
    direction = torch.tensor(np.concatenate([np.asarray(c["direction"], np.uint8)
                                             for c in cases]), device="cuda")
    ready = torch.tensor(np.concatenate([np.asarray(c["ready"], np.int64) for c in cases]),
                         device="cuda")
    delivered, res = link_batch(as_profiles(cases), offsets, direction, ready)
    d = delivered.cpu().numpy().view(np.uint64)
    return [d[offsets[k]:offsets[k + 1]] for k in range(len(cases))], res


def test_reference_links():
    cases = json.loads(GOLDEN.read_text())
    delivered, res = run(cases)
    for k, c in enumerate(cases):
        assert res[k]["status"] == 0, k
        assert delivered[k].tolist() == c["delivered"], k
        assert res[k]["counters"].tolist() == c["counters"], k
        assert [int(res[k]["ar_credits"]), int(res[k]["r_credits"]), int(res[k]["now"])] == \
            c["tail"], k


def random_cases(rng, n):
    cases = []
    for _ in range(n):
        prof = {"gt": int(rng.choice([8, 16, 32])), "ar": int(rng.choice([3, 4, 12, 40, 128])),
                "r": int(rng.choice([14, 20, 56, 200])),
                "accepted": int(rng.choice([1, 2, 4, 16, 128])),
                "prop": int(rng.choice([0, 1, 7, 100])),
                "consume": [int(rng.choice([0, 0, 3, 50])), int(rng.choice([0, 2, 100, 1000]))]}
        m = int(rng.integers(1, 3000))
        direction = (rng.random(m) < rng.random()).astype(np.uint8)
        gaps = np.where(rng.random(m) < rng.random(), 0, rng.integers(0, 40, m))
        cases.append({"profile": prof, "direction": direction,
                      "ready": np.cumsum(gaps).astype(np.uint64)})
    return cases


def test_many_links_match_oracle():
    rng = np.random.default_rng(8)
    cases = random_cases(rng, 400)
    delivered, res = run(cases)
    for k, c in enumerate(cases):
        want = ho.link_run(c["profile"], c["direction"], c["ready"])
        assert res[k]["status"] == 0
        assert np.array_equal(delivered[k], want[0]), k
        assert res[k]["counters"].tolist() == want[1].tolist(), k
        assert [int(res[k]["now"]), int(res[k]["ar_credits"]), int(res[k]["r_credits"])] == \
            list(want[2:]), k


def test_out_of_order_link_and_bad_profile():
    rng = np.random.default_rng(9)
    cases = random_cases(rng, 3)
    cases[1]["ready"] = cases[1]["ready"][::-1].copy()  # decreasing: that link is refused
    if cases[1]["ready"].size == 1:
        cases[1]["ready"] = np.array([5, 1], np.uint64)
        cases[1]["direction"] = np.array([0, 0], np.uint8)
    delivered, res = run(cases)
    assert res[1]["status"] != 0
    for k in (0, 2):
        want = ho.link_run(cases[k]["profile"], cases[k]["direction"], cases[k]["ready"])
        assert res[k]["status"] == 0 and np.array_equal(delivered[k], want[0])
    bad = dict(cases[0])
    bad["profile"] = dict(cases[0]["profile"], gt=64)
    with pytest.raises(HbfsimError):
        run([bad])


def _linked_gpu(tmp, stacks, arrays, profile):
    from helpers import Setup, make_context, to_device
    from hbfsim_b200 import submit_linked
    from hbfsim_b200 import workloads as wl
    p = wl.c0_profile()
    s = Setup(profile=p, model=3, stacks=stacks, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, p["capacity_bytes"] - (1 << 20), 1, 3)]
    ctx = make_context(s, tmp)
    dev = to_device(arrays)
    profs = link_profiles(stacks, profile["gt"], profile["ar"], profile["r"],
                          profile["accepted"], profile["prop"], [profile["consume"]] * stacks)
    out, die, res, ar = submit_linked(ctx, *dev, profs, stacks)
    got = (out.done_ns.cpu().numpy().view(np.uint64), die.done_ns.cpu().numpy().view(np.uint64),
           out.status.cpu().numpy(), ar.cpu().numpy())
    assert (res["status"] == 0).all()
    ctx.close()
    return s, got


def test_linked_stage_against_reference_link(tmp_path):
    """Accesses through the die model and then their stack's UCIe link (AR
    at the arrival, R at the die completion): every R and AR delivery equal
    to the reference StreamingLink's on the same messages
    (tests/golden/linked_goldens.json)."""
    from hbfsim_b200 import workloads as wl
    g = json.loads((GOLDEN.parent / "linked_goldens.json").read_text())
    p = wl.c0_profile()
    arrays = wl.c0_trace(g["n"], seed=g["seed"], range_length=p["capacity_bytes"] - (1 << 20))
    _, (linked, done, status, ar) = _linked_gpu(str(tmp_path), g["stacks"], arrays,
                                                g["profile"])
    assert done.tolist() == g["die_done"]
    assert status.tolist() == g["status"]
    assert linked.tolist() == g["linked_done"]
    assert ar.tolist() == g["ar_delivered"]


def test_linked_stage_matches_oracle(tmp_path):
    """A larger trace on 4 stacks (4 links), against the oracle's die model
    and link composed the same way."""
    from helpers import OracleRun, oracle_linked
    from hbfsim_b200 import workloads as wl
    p = wl.c0_profile()
    arrays = wl.c0_trace(120_000, seed=8, range_length=p["capacity_bytes"] - (1 << 20))
    profile = {"gt": 32, "ar": 12, "r": 56, "accepted": 8, "prop": 3, "consume": [0, 5]}
    s, (linked, done, status, ar) = _linked_gpu(str(tmp_path), 4, arrays, profile)
    want = oracle_linked(s, OracleRun(s), arrays, profile)
    assert np.array_equal(done, want[1])
    assert np.array_equal(status, want[2])
    bad = np.flatnonzero(linked != want[0])
    assert bad.size == 0, f"linked completion differs at {bad[:5]}"
    assert np.array_equal(ar, want[3])
    assert (linked >= done).all()
