// The FS-L top-P pool as a sorted list (ceiling descending, cell index ascending) held in shared memory and maintained
// by one warp. Cells only ever join the ranking (a completed cell's ceiling is fixed), so the top-P of a longer prefix
// is the top-P of (previous top-P + new cells): one sorted insert per new cell.
#pragma once
#include "common.cuh"

// Insert cell (cv, ci) into the list lc/li of n entries with capacity P. All 32 lanes call it; n is updated uniformly.
__device__ __forceinline__ void pool_list_insert(float* lc, int* li, int& n, int P, float cv, int ci, int lane) {
    // fast reject: list full and the new cell ranks after its last entry
    if (n == P && !pool_before(cv, ci, lc[P - 1], li[P - 1])) return;
    int cnt = 0;
    for (int p = lane; p < n; p += 32) cnt += pool_before(lc[p], li[p], cv, ci) ? 1 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(FS_FULL, cnt, o);
    const int ins = cnt;
    if (ins >= P) return;
    const int nn = (n + 1 < P) ? n + 1 : P;
    // shift [ins, nn-1) right by one: read everything first, then write
    float tv[FSATTN_MAX_POOL / 32];
    int ti[FSATTN_MAX_POOL / 32];
#pragma unroll
    for (int j = 0; j < FSATTN_MAX_POOL / 32; j++) {
        const int p = lane + 32 * j;
        if (p > ins && p < nn) { tv[j] = lc[p - 1]; ti[j] = li[p - 1]; }
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < FSATTN_MAX_POOL / 32; j++) {
        const int p = lane + 32 * j;
        if (p > ins && p < nn) { lc[p] = tv[j]; li[p] = ti[j]; }
        else if (p == ins) { lc[p] = cv; li[p] = ci; }
    }
    __syncwarp();
    n = nn;
}
