// thermal.cu -- eq3 layered thermal grid on the GPU (placeholder entry points).
#include "context.h"

namespace hbfb {
struct ThermalState {
    int unused;
};
void thermal_destroy(ThermalState* t) { delete t; }
}  // namespace hbfb

extern "C" {
int hbfsim_thermal_configure_v1(hbfsim_context* c, const hbfsim_thermal_config_v1* cfg)
{
    return (!c || !cfg) ? HBFSIM_INVALID_ARGUMENT : HBFSIM_UNSUPPORTED;
}
int hbfsim_advance_epoch_v1(hbfsim_context* c, double, void*)
{
    return !c ? HBFSIM_INVALID_ARGUMENT : HBFSIM_UNSUPPORTED;
}
int hbfsim_get_temperatures_v1(hbfsim_context* c, double*, uint64_t)
{
    return !c ? HBFSIM_INVALID_ARGUMENT : HBFSIM_UNSUPPORTED;
}
int hbfsim_get_die_temperatures_v1(hbfsim_context* c, double*, uint64_t)
{
    return !c ? HBFSIM_INVALID_ARGUMENT : HBFSIM_UNSUPPORTED;
}
}
