// Head-sharded decode: the exchange of a layer's head outputs between the GPUs of a box as ONE small kernel per rank over
// peer memory, instead of a library all-gather (about 10 us of launch + protocol latency for 1 - 3 KB per step and layer).
//
// Every rank owns a slab (cudaMalloc, exported once with a CUDA IPC handle and opened by its peers) holding receive
// buffers of 8-byte words {4 bytes of data, 4 bytes of flag}: ll[slot][parity][source rank][word]. A call of rank r for
// slot s takes its call count e (kept on the device, so a captured graph replays the same launch every step) and
//   1. stores every 4 bytes of its rows (B, dl) together with e as ONE 8-byte word into ll[s][e & 1][r] of every peer
//      (an 8-byte store arrives whole, so data and flag need no fence between them and no second message), and copies
//      the rows into its own columns of the local gathered buffer y_out (B, world dl);
//   2. polls the words of ll[s][e & 1][p] in its OWN slab for every peer p until their flag equals e, and writes their
//      data into p's columns of y_out.
// A word is overwritten by the call e + 2 of the same slot; its sender gets there only after this rank has posted call
// e + 1 of that slot, i.e. after it has read call e. The polls are bounded by the global timer: when one runs out the
// kernel raises bit p of *status and returns. No load ever targets a peer's memory, nothing is multicast, and no kernel
// of one GPU waits for another kernel of the SAME GPU.
#include "common.cuh"

namespace {

struct PeerArgs {
    const uint32_t* y_local;
    uint32_t* y_out;
    uint2* ll_dst[FSATTN_PEER_MAX];
    int32_t* epoch;
    int32_t* status;
    int B, dl2, rank, world, slot;
    int64_t timeout_ns;
};

__device__ __forceinline__ uint64_t peer_now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr int PEER_THREADS = 256;
constexpr int PEER_U = 4;

__global__ void __launch_bounds__(PEER_THREADS) peer_gather_kernel(PeerArgs a) {
    const int tid = threadIdx.x;
    const int e = a.epoch[a.slot] + 1;                                // written by this kernel's previous call only
    asm volatile("griddepcontrol.wait;" ::: "memory");               // the attention step that wrote y_local
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the consumer may start streaming its weights
    const int n = a.B * a.dl2;                                        // 4-byte words of this rank's rows
    const int64_t buf = ((int64_t)(a.slot * 2 + (e & 1)) * a.world) * n;
    const int row = a.world * a.dl2;
    // 1. my rows: to every peer's receive buffer with the flag, and into my own columns of y_out
    for (int i0 = tid; i0 < n; i0 += PEER_THREADS * PEER_U) {
        uint32_t v[PEER_U];
#pragma unroll
        for (int u = 0; u < PEER_U; ++u) { const int i = i0 + u * PEER_THREADS; v[u] = i < n ? a.y_local[i] : 0u; }
#pragma unroll
        for (int u = 0; u < PEER_U; ++u) {
            const int i = i0 + u * PEER_THREADS;
            if (i >= n) break;
            for (int p = 0; p < a.world; ++p) {
                if (p == a.rank) continue;
                uint2* w = a.ll_dst[p] + buf + (int64_t)a.rank * n + i;
                asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(w), "r"(v[u]), "r"(e) : "memory");
            }
            const int b = i / a.dl2, c = i - b * a.dl2;
            a.y_out[(int64_t)b * row + a.rank * a.dl2 + c] = v[u];
        }
    }
    // 2. the peers' rows out of my own receive buffers
    const uint64_t t0 = peer_now_ns();
    const int items = (a.world - 1) * n;
    for (int j = tid; j < items; j += PEER_THREADS) {
        int p = j / n;
        const int i = j - p * n;
        if (p >= a.rank) ++p;
        const uint2* w = a.ll_dst[a.rank] + buf + (int64_t)p * n + i;
        uint32_t x, f;
        bool ok = true;
        for (;;) {
            asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(x), "=r"(f) : "l"(w) : "memory");
            if ((int)f == e) break;
            if ((int64_t)(peer_now_ns() - t0) > a.timeout_ns) { ok = false; break; }
        }
        if (!ok) {
            atomicOr(a.status, 1 << p);
            break;
        }
        const int b = i / a.dl2, c = i - b * a.dl2;
        a.y_out[(int64_t)b * row + p * a.dl2 + c] = x;
    }
    if (tid == 0) a.epoch[a.slot] = e;
}

}  // namespace

extern "C" int64_t fsattn_peer_ll_bytes(int32_t B, int32_t dl, int32_t world, int32_t n_slots) {
    if (B <= 0 || dl <= 0 || world <= 0 || n_slots <= 0) return 0;
    return (int64_t)n_slots * 2 * world * ((int64_t)B * dl / 2) * 8;
}

extern "C" int fsattn_peer_gather(const fsattn_peer_gather_t* g, fsattn_stream_t stream) {
    FS_REQUIRE(g && g->y_local && g->y_out && g->epoch && g->status, "peer_gather: null argument");
    FS_REQUIRE(g->world >= 1 && g->world <= FSATTN_PEER_MAX && g->rank >= 0 && g->rank < g->world, "peer_gather: rank %d of %d (at most %d ranks)",
               g->rank, g->world, FSATTN_PEER_MAX);
    FS_REQUIRE(g->B > 0 && g->dl > 0 && g->dl % 2 == 0 && g->slot >= 0, "peer_gather: B = %d rows of dl = %d elements (even)", g->B, g->dl);
    FS_REQUIRE((int64_t)g->B * g->dl <= (1 << 20), "peer_gather: at most 2^20 elements per call");
    FS_REQUIRE(g->timeout_ns > 0 && g->timeout_ns <= 2000000000ll, "peer_gather: timeout_ns in (0, 2e9]");
    FS_REQUIRE(((uintptr_t)g->y_local & 3) == 0 && ((uintptr_t)g->y_out & 3) == 0, "peer_gather: rows must be 4-byte aligned");
    PeerArgs a;
    a.y_local = (const uint32_t*)g->y_local;
    a.y_out = (uint32_t*)g->y_out;
    for (int p = 0; p < FSATTN_PEER_MAX; ++p) {
        a.ll_dst[p] = p < g->world ? (uint2*)g->ll_dst[p] : nullptr;
        if (p < g->world) FS_REQUIRE(g->ll_dst[p] && ((uintptr_t)g->ll_dst[p] & 7) == 0, "peer_gather: receive buffer of rank %d null or unaligned", p);
    }
    a.epoch = g->epoch;
    a.status = g->status;
    a.B = g->B; a.dl2 = g->dl / 2; a.rank = g->rank; a.world = g->world; a.slot = g->slot;
    a.timeout_ns = g->timeout_ns;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(PEER_THREADS);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g->pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, peer_gather_kernel, a);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("peer_gather: launch failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

// ---- the slab and its handle ---------------------------------------------------------------------------------------
extern "C" int fsattn_peer_alloc(int64_t bytes, void** ptr) {
    FS_REQUIRE(ptr && bytes > 0, "peer_alloc: null pointer or bad size");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        if (p) cudaFree(p);
        fs_set_error("peer_alloc: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    *ptr = p;
    return FSATTN_OK;
}

extern "C" int fsattn_peer_free(void* ptr) {
    if (ptr && cudaFree(ptr) != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("peer_free: cudaFree failed");
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

extern "C" int fsattn_peer_export(void* ptr, uint8_t* handle) {
    FS_REQUIRE(ptr && handle, "peer_export: null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == FSATTN_PEER_HANDLE_BYTES, "handle size");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("peer_export: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    memcpy(handle, &h, sizeof(h));
    return FSATTN_OK;
}

extern "C" int fsattn_peer_open(const uint8_t* handle, void** ptr) {
    FS_REQUIRE(ptr && handle, "peer_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("peer_open: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    *ptr = p;
    return FSATTN_OK;
}

extern "C" int fsattn_peer_close(void* ptr) {
    if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("peer_close: cudaIpcCloseMemHandle failed");
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}
