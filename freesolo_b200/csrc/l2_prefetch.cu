// Pull a byte range into L2 ahead of its use (decode-step weights of the layers to come). One bulk prefetch instruction
// per 16 KB piece; nothing is written, nothing is waited for.
#include "common.cuh"

namespace {

constexpr int PF_CHUNK = 16 * 1024;

__global__ void __launch_bounds__(128) l2_prefetch_kernel(const char* base, int64_t bytes) {
    const int64_t nchunk = (bytes + PF_CHUNK - 1) / PF_CHUNK;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nchunk; c += (int64_t)gridDim.x * blockDim.x) {
        const int64_t off = c * PF_CHUNK;
        const uint32_t n = (uint32_t)min((int64_t)PF_CHUNK, bytes - off) & ~15u;      // multiples of 16 bytes
        if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"(n) : "memory");
    }
}

}  // namespace

extern "C" int fsattn_l2_prefetch(const void* ptr, int64_t bytes, fsattn_stream_t stream) {
    FS_REQUIRE(ptr != nullptr && bytes >= 0, "l2_prefetch: null pointer or negative size");
    FS_REQUIRE(((uintptr_t)ptr & 15) == 0, "l2_prefetch: the range must start on a 16-byte boundary");
    if (bytes < 16) return FSATTN_OK;
    const int64_t nchunk = (bytes + PF_CHUNK - 1) / PF_CHUNK;
    const int grid = (int)min((int64_t)32, (nchunk + 127) / 128);
    l2_prefetch_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>((const char*)ptr, bytes);
    return fs_check_launch("l2_prefetch_kernel");
}
