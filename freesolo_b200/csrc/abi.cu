// Host side of the C ABI: error text, device setup and the entry points that only dispatch.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

static thread_local char g_err[512] = "";

void fs_set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int fs_check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fs_set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

int fs_window_prefill_simt(const fsattn_window_prefill_t* a, cudaStream_t st);
int fs_window_prefill_tc(const fsattn_window_prefill_t* a, cudaStream_t st);
bool fs_window_prefill_tc_ok(const fsattn_window_prefill_t* a);

extern "C" int fsattn_version(void) { return 1; }

extern "C" const char* fsattn_last_error(void) { return g_err; }

extern "C" int fsattn_init(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        fs_set_error("fsattn_init: no CUDA device %d", device);
        return FSATTN_EINVAL;
    }
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess) {
        fs_set_error("fsattn_init: cannot query device %d", device);
        return FSATTN_ELAUNCH;
    }
    if (p.major != 10) {
        fs_set_error("fsattn_init: device %d is sm_%d%d; this library is built for sm_100a only", device, p.major, p.minor);
        return FSATTN_EUNSUPPORTED;
    }
    return FSATTN_OK;
}

extern "C" int fsattn_window_prefill(const fsattn_window_prefill_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->q.ptr && a->k.ptr && a->v.ptr && a->cos && a->sin && a->out, "window_prefill: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->N > 0 && a->W >= 0 && a->pos0 >= 0, "window_prefill: bad sizes");
    FS_UNSUPPORTED(a->D != 64 && a->D != 96 && a->D != 128, "window_prefill: head_dim %d not in {64,96,128}", a->D);
    const fsattn_bhnd_t* t[3] = {&a->q, &a->k, &a->v};
    for (int i = 0; i < 3; i++)
        FS_REQUIRE(((uintptr_t)t[i]->ptr & 15) == 0 && t[i]->sn % 8 == 0 && t[i]->sh % 8 == 0 && t[i]->sb % 8 == 0,
                   "window_prefill: Q, K and V rows must be 16-byte aligned");
    FS_REQUIRE(((uintptr_t)a->cos & 15) == 0 && ((uintptr_t)a->sin & 15) == 0 && ((uintptr_t)a->out & 15) == 0,
               "window_prefill: tables and output must be 16-byte aligned");
    FS_REQUIRE(a->impl == 0 || a->impl == 1, "window_prefill: impl %d", a->impl);
    cudaStream_t st = (cudaStream_t)stream;
    if (a->impl == 0 && fs_window_prefill_tc_ok(a)) return fs_window_prefill_tc(a, st);
    return fs_window_prefill_simt(a, st);
}
