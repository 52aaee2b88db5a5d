// Tensor-core (tcgen05 / TMEM / TMA) window attention for prefill. Placeholder dispatch until the kernel lands: reports
// that no shape is covered, so every call takes the CUDA-core kernel.
#include "common.cuh"

bool fs_window_prefill_tc_ok(const fsattn_window_prefill_t*) { return false; }
int fs_window_prefill_tc(const fsattn_window_prefill_t*, cudaStream_t) {
    fs_set_error("window_prefill: tensor-core kernel not built");
    return FSATTN_EUNSUPPORTED;
}
