// FS-B prefill beams for whole 128-query blocks: four THREADS per query, and the node scores of the block from tensor-core tiles.
// (Included by fsb_select.cu inside its namespace: it uses SpineSm, build_spine, count_below, SelArgs and the node refs.)
//
// The queries of one block walk almost the same part of the forest: their 2048 frontier slots hold a few dozen distinct
// nodes per level. So a level is scored once for the block: every query lists the children of its frontier, the distinct
// chunk nodes among them are collected in a shared hash set (one insert per distinct node of a warp), their bf16 mean rows
// are staged 64 at a time and multiplied with the block's 128 queries on mma.sync.m16n8k16 tiles (exact products, fp32
// accumulation), and each query then reads the dot products of ITS children from shared memory, adds radius and
// position terms, ranks its 32 children ((score desc, position asc), the order of the one-warp-per-query kernel) and
// rebuilds its frontier: carried leaves first in slot order, then the kept children. Spine nodes (fp32 means, one chain per
// forest) are scored by the query itself. A query is a quad of neighbouring lanes: each owns four frontier slots and
// their eight children in REGISTERS (every loop over them is unrolled, no indexed local arrays; the loop over the three
// partner lanes is a real loop, which keeps the level's code small enough for the instruction cache), the quad exchanges
// scores by shuffles, and the new frontier goes through a shared-memory row laid out [slot][query], which any slot
// index reaches without bank conflicts. Any number of distinct nodes is handled (up to 128 x 32, in 64-column passes);
// the few-dozen case is the fast one.

constexpr int BK_CT = 64;            // distinct nodes scored per pass (columns of the score tile)
constexpr int BK_HT = 4096;          // hash slots = the most distinct children a level can have (128 queries x 32)
constexpr int BK_THREADS = 512;
constexpr int BK_SLD = BK_CT + 2;    // row pitch of the score tile in floats
constexpr int BK_T = 4;              // threads per query
constexpr int BK_HS = WMAX / BK_T;   // frontier slots per thread

template <int D>
struct BeamSmem {
    static constexpr int PITCH = D * 2 + 16;                            // staged mean row: conflict-free fragment reads
    static constexpr size_t HKEY = 0;                                   // int[BK_HT]: node ref or -1
    static constexpr size_t HIDX = HKEY + (size_t)BK_HT * 4;            // uint16[BK_HT]: column of the slot's node
    static constexpr size_t ULIST = HIDX + (size_t)BK_HT * 2;           // uint16[BK_HT]: column -> slot
    static constexpr size_t MU = ULIST + (size_t)BK_HT * 2;
    static constexpr size_t AUX = MU + (size_t)BK_CT * PITCH;           // float4[BK_CT]
    static constexpr size_t SC = AUX + (size_t)BK_CT * 16;              // float[128][BK_SLD]
    static constexpr size_t FREF = SC;                                  // int[WMAX][128]: the new frontier's refs; lies over
    static constexpr size_t FMETA = FREF + (size_t)WMAX * 128 * 4;      // int[WMAX][128]   the score tile (used after it)
    static constexpr size_t TOTAL = SC + (size_t)128 * BK_SLD * 4;
};

__device__ __forceinline__ void bk_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// slot of `ref` in the open-addressing set; a new ref is appended to the level's list (its slot in ulist, its column in
// hidx - both read only after the block barrier that follows the inserts). At most BK_HT distinct refs are ever offered.
__device__ __forceinline__ uint32_t bk_hash(int ref) { return ((uint32_t)ref * 2654435761u) >> 20; }        // 12 bits
__device__ __forceinline__ int bk_insert(int* hkey, unsigned short* hidx, unsigned short* ulist, int* ucount, int ref) {
    uint32_t h = bk_hash(ref);
    for (int probe = 0; probe < BK_HT; ++probe) {
        const int old = atomicCAS(&hkey[h], -1, ref);
        if (old == -1) {
            const int idx = atomicAdd(ucount, 1);
            hidx[h] = (unsigned short)idx;
            ulist[idx] = (unsigned short)h;
            break;
        }
        if (old == ref) break;
        h = (h + 1) & (BK_HT - 1);
    }
    return (int)h;
}

// position term of a node score: lam * amax * erf(|qpos - centre| / (2 sigma)); erf is 1 in fp32 from 4 on
__device__ __forceinline__ float bk_score(float dot_scaled, float qn, float rad, float am, int pm, float qpos, float lam,
                                          float inv_two_sig, float scale) {
    const float content = f_add(dot_scaled, f_mul(f_mul(qn, rad), scale));
    const float ppos = f_mul(f_add((float)pm, 0.5f), 32.0f);
    const float xe = f_mul(fabsf(f_add(qpos, -ppos)), inv_two_sig);
    const float e = (xe < 4.0f) ? erff(xe) : 1.0f;
    return f_add(content, f_mul(f_mul(lam, am), e));
}

// score of a spine node (fp32 mean in shared memory) for one query; rare (one chain per forest), so kept out of line
template <int D>
__device__ __noinline__ float bk_spine_score(const float* x, const bf16* qrow, float qn, float qpos, float lam, float inv_two_sig,
                                             float scale) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int v = 0; v < D / 8; ++v) {
        const uint4 w = *(const uint4*)(qrow + v * 8);
        const float* xx = x + v * 8;
        s0 = fmaf(bf_lo(w.x), xx[0], s0); s1 = fmaf(bf_hi(w.x), xx[1], s1);
        s2 = fmaf(bf_lo(w.y), xx[2], s2); s3 = fmaf(bf_hi(w.y), xx[3], s3);
        s0 = fmaf(bf_lo(w.z), xx[4], s0); s1 = fmaf(bf_hi(w.z), xx[5], s1);
        s2 = fmaf(bf_lo(w.w), xx[6], s2); s3 = fmaf(bf_hi(w.w), xx[7], s3);
    }
    return bk_score(f_mul((s0 + s1) + (s2 + s3), scale), qn, x[D], x[D + 1], __float_as_int(x[D + 2]), qpos, lam, inv_two_sig, scale);
}

template <int D>
__global__ void __launch_bounds__(BK_THREADS, 2) fsb_beam_block_kernel(SelArgs A) {
    using SM = BeamSmem<D>;
    constexpr int KS = D / 16;                   // k-steps of a 16 x 8 tile
    constexpr int CH = D / 8;                    // 16-byte chunks of a mean row
    constexpr int NC = 2 * BK_HS;                // children per thread
    const fsattn_fsb_select_t& a = A.a;
    const int blk = blockIdx.x, t = blockIdx.y;
    const int b = t / A.H, hd = t % A.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qi = tid >> 2, sub = tid & 3;      // query of this thread; which four frontier slots it owns
    extern __shared__ __align__(16) unsigned char dsm[];
    int* hkey = (int*)(dsm + SM::HKEY);
    unsigned short* hidx = (unsigned short*)(dsm + SM::HIDX);
    unsigned short* ulist = (unsigned short*)(dsm + SM::ULIST);
    unsigned char* smu = dsm + SM::MU;
    float4* saux = (float4*)(dsm + SM::AUX);
    float* ssc = (float*)(dsm + SM::SC);
    int* frs_ref = (int*)(dsm + SM::FREF) + qi;          // [slot * 128]
    int* frs_meta = (int*)(dsm + SM::FMETA) + qi;
    __shared__ SpineSm<D> sp;
    __shared__ BeamPre pre;
    __shared__ int ucount;

    const float lam = a.lam[hd], sig = a.sigma[hd];
    const float inv_two_sig = f_div(1.0f, f_mul(2.0f, sig));
    const int Wc = a.width + a.width2;
    const int nq = min(a.Bq, a.N - blk * a.Bq);
    const int E = (a.q_pos0 + blk * a.Bq) / 32;
    const bf16* qbase = (const bf16*)a.q.ptr + b * a.q.sb + hd * a.q.sh + (int64_t)blk * a.Bq * a.q.sn;
    const bool isq = qi < nq;
    const bf16* qrow = qbase + (int64_t)(isq ? qi : 0) * a.q.sn;
    const int mg = lane >> 2, mt = lane & 3;     // MMA fragment coordinates
    const int mr0 = (warp & 7) * 16 + mg, mr1 = mr0 + 8;     // warps w and w + 8 share 16 query rows and split the column tiles

    // ---- per query: position and radius factor ||q|| coef (sum of squares in the halving order of the warp kernel) ----
    const float qpos = (float)(a.q_pos0 + blk * a.Bq + qi);
    float qn;
    {
        float p[FsbDim<D>::DP];
#pragma unroll
        for (int v = 0; v < CH; ++v) {
            const uint4 w = *(const uint4*)(qrow + v * 8);
            const float x[8] = {bf_lo(w.x), bf_hi(w.x), bf_lo(w.y), bf_hi(w.y), bf_lo(w.z), bf_hi(w.z), bf_lo(w.w), bf_hi(w.w)};
#pragma unroll
            for (int j = 0; j < 8; ++j) p[v * 8 + j] = f_mul(x[j], x[j]);
        }
#pragma unroll
        for (int d = D; d < FsbDim<D>::DP; ++d) p[d] = 0.f;
        qn = f_mul(f_sqrt(fsb_thread_det_sum<D>(p)), a.radius_coef);
    }
    for (int i = tid; i < BK_HT; i += BK_THREADS) hkey[i] = -1;
    if (tid == 0) ucount = 0;

    int cells[2][BK_HS];
    int nv = 0;                                  // children this thread scored (the quad's sum is the query's count)
#pragma unroll
    for (int f = 0; f < 2; ++f)
#pragma unroll
        for (int j = 0; j < BK_HS; ++j) cells[f][j] = -1;

    const int nbeam = a.width2 > 0 ? 2 : 1;
    for (int f = 0; f < nbeam; ++f) {
        const fsattn_fsb_forest_t& F = f == 0 ? a.main : a.second;
        const int width = f == 0 ? a.width : a.width2;
        __syncthreads();
        if (warp == 0) {
            const int m_b = count_below(F.adm + (int64_t)t * F.m_cap, F.m_tot[t], E);
            build_spine<D>(F, t, m_b, sp, lane);
            __syncwarp();
            beam_prefix<D>(F, t, sp, width, lane, pre);
        }
        __syncthreads();
        const int64_t nrow = (int64_t)t * fsb_nodes_per_row(F.m_cap, F.compact);
        const bf16* node_mu = (const bf16*)F.node_mu + nrow * D;
        const float4* aux = (const float4*)F.node_aux + nrow;
        const int root = sp.root;
        if (root == -1) continue;                 // no admitted cell is visible to this block (the same for every thread)
        const int d0 = sp.height;
        const int W = min(width, (d0 >= 5) ? 32 : (1 << d0));

        // one child of this thread: a chunk node goes into the block's set (cx = its slot), a spine node is scored here.
        // Most nodes are already in the set when a warp offers them (another warp, or an earlier child): one plain read of the
        // home slot finds those; the rest take the slow path, one insert per distinct node of the warp.
        auto place = [&](int cref, int c, int (&cx)[NC], unsigned& spm) {
            const int key = cref >= 0 ? cref : -1;
            const uint32_t h0 = bk_hash(key);
            const bool hit = key < 0 || *(volatile int*)&hkey[h0] == key;
            int slot = (int)h0;
            if (__any_sync(FS_FULL, !hit)) {
                const int k2 = hit ? -1 : key;
                const unsigned grp = __match_any_sync(FS_FULL, k2);
                const int leader = __ffs(grp) - 1;
                int s2 = 0;
                if (k2 >= 0 && lane == leader) s2 = bk_insert(hkey, hidx, ulist, &ucount, k2);
                s2 = __shfl_sync(FS_FULL, s2, leader);
                if (!hit) slot = s2;
            }
            cx[c] = slot;
            if (cref < -1) {
                cx[c] = __float_as_int(bk_spine_score<D>(sp.node[-cref - 2], qrow, qn, qpos, lam, inv_two_sig, a.scale));
                spm |= 1u << c;
            }
        };
        // scores of the children in vm that are chunk nodes (after the block barrier that follows their inserts): the level's
        // distinct nodes, BK_CT per pass, staged, multiplied with the 128 queries, read back per child
        auto score_level = [&](int (&cx)[NC], unsigned vm, unsigned spm) {
            const int U = ucount;
            unsigned pend = vm & ~spm;
#pragma unroll
            for (int c = 0; c < NC; ++c)
                if ((pend >> c) & 1) cx[c] = hidx[cx[c]];
            for (int p0 = 0; p0 < U; p0 += BK_CT) {
                const int ncol = min(BK_CT, U - p0);
                for (int i = tid; i < BK_CT * CH; i += BK_THREADS) {
                    const int r = i / CH, v = i % CH;
                    uint4 w = make_uint4(0u, 0u, 0u, 0u);
                    if (r < ncol) w = *(const uint4*)(node_mu + (int64_t)REF_ID(hkey[ulist[p0 + r]]) * D + v * 8);
                    *(uint4*)(smu + (size_t)r * SM::PITCH + v * 16) = w;
                }
                if (tid < ncol) saux[tid] = aux[REF_ID(hkey[ulist[p0 + tid]])];
                uint32_t afr[KS][4];              // this warp's 16 query rows (L1-resident after the first pass)
                {
                    const bf16* q0 = qbase + (int64_t)mr0 * a.q.sn;
                    const bf16* q1 = qbase + (int64_t)mr1 * a.q.sn;
#pragma unroll
                    for (int kk = 0; kk < KS; ++kk) {
                        afr[kk][0] = mr0 < nq ? *(const uint32_t*)(q0 + kk * 16 + 2 * mt) : 0u;
                        afr[kk][1] = mr1 < nq ? *(const uint32_t*)(q1 + kk * 16 + 2 * mt) : 0u;
                        afr[kk][2] = mr0 < nq ? *(const uint32_t*)(q0 + kk * 16 + 8 + 2 * mt) : 0u;
                        afr[kk][3] = mr1 < nq ? *(const uint32_t*)(q1 + kk * 16 + 8 + 2 * mt) : 0u;
                    }
                }
                __syncthreads();
                if (tid == 0) ucount = 0;         // every thread has read U
                {
                    const int ntile = (ncol + 7) >> 3;
                    for (int nt = warp >> 3; nt < ntile; nt += 2) {
                        float c[4] = {0.f, 0.f, 0.f, 0.f};
                        const unsigned char* br = smu + (size_t)(nt * 8 + mg) * SM::PITCH + mt * 4;
#pragma unroll
                        for (int kk = 0; kk < KS; ++kk) {
                            const uint32_t b0 = *(const uint32_t*)(br + kk * 32);
                            const uint32_t b1 = *(const uint32_t*)(br + kk * 32 + 16);
                            bk_mma(c, afr[kk], b0, b1);
                        }
                        float* d0p = ssc + (size_t)mr0 * BK_SLD + nt * 8 + 2 * mt;
                        *(float2*)d0p = make_float2(c[0], c[1]);
                        *(float2*)(d0p + 8 * BK_SLD) = make_float2(c[2], c[3]);
                    }
                }
                __syncthreads();
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const unsigned j = (unsigned)(cx[c] - p0);
                    if (((pend >> c) & 1) && j < (unsigned)BK_CT) {
                        const float4 ax = saux[j];
                        cx[c] = __float_as_int(bk_score(f_mul(ssc[(size_t)qi * BK_SLD + j], a.scale), qn, ax.x, ax.y,
                                                        __float_as_int(ax.z), qpos, lam, inv_two_sig, a.scale));
                        pend &= ~(1u << c);
                    }
                }
                if (p0 + BK_CT >= U)              // last pass: empty the set for the next level
                    for (int i = tid; i < U; i += BK_THREADS) hkey[ulist[i]] = -1;
                __syncthreads();
            }
        };

        int fref[BK_HS], fmeta[BK_HS];            // this thread's frontier slots BK_HS * sub + j (the frontier is compact)
#pragma unroll
        for (int j = 0; j < BK_HS; ++j) { fref[j] = -1; fmeta[j] = 0; }
        if (pre.rounds > 0) {
            // ---- the block's query-independent head (the rounds whose children all fit in the frontier): its nodes are
            // scored once and put into this query's order - older rounds first, a round's nodes by score ----
            int cx[NC];
            unsigned vm = 0, spm = 0;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int idx = BK_HS * sub + c;
                const bool valid = c < BK_HS && isq && idx < pre.n;
                vm |= (valid ? 1u : 0u) << c;
                place(valid ? pre.ref[idx] : -1, c, cx, spm);
            }
            __syncthreads();
            score_level(cx, vm, spm);
            float sc[BK_HS];
            int rn[BK_HS], rank[BK_HS];
#pragma unroll
            for (int c = 0; c < BK_HS; ++c) {
                const bool valid = (vm >> c) & 1;
                sc[c] = valid ? __int_as_float(cx[c]) : FS_NEG_SCORE;
                rn[c] = valid ? pre.rnd[BK_HS * sub + c] : (1 << 20);
                rank[c] = 0;
            }
#pragma unroll
            for (int i = 0; i < BK_HS; ++i)
#pragma unroll
                for (int k = i + 1; k < BK_HS; ++k) {
                    const bool first = rn[i] < rn[k] || (rn[i] == rn[k] && sc[i] >= sc[k]);
                    rank[k] += first ? 1 : 0;
                    rank[i] += first ? 0 : 1;
                }
#pragma unroll 1
            for (int p = 1; p < BK_T; ++p) {
                const bool plow = (sub ^ p) < sub;
#pragma unroll
                for (int o = 0; o < BK_HS; ++o) {
                    const float po = __shfl_xor_sync(FS_FULL, sc[o], p);
                    const int pr = __shfl_xor_sync(FS_FULL, rn[o], p);
#pragma unroll
                    for (int c = 0; c < BK_HS; ++c)
                        rank[c] += (pr < rn[c] || (pr == rn[c] && (po > sc[c] || (plow && po == sc[c])))) ? 1 : 0;
                }
            }
#pragma unroll
            for (int j = 0; j < BK_HS; ++j) { frs_ref[(BK_HS * sub + j) * 128] = -1; frs_meta[(BK_HS * sub + j) * 128] = 0; }
            __syncwarp();
#pragma unroll
            for (int c = 0; c < BK_HS; ++c) {
                if ((vm >> c) & 1) {
                    frs_ref[rank[c] * 128] = pre.ref[BK_HS * sub + c];
                    frs_meta[rank[c] * 128] = pre.meta[BK_HS * sub + c];
                }
            }
            __syncwarp();
#pragma unroll
            for (int j = 0; j < BK_HS; ++j) { fref[j] = frs_ref[(BK_HS * sub + j) * 128]; fmeta[j] = frs_meta[(BK_HS * sub + j) * 128]; }
            __syncwarp();
            if (isq && sub == 0) nv += pre.nvis;
        } else if (isq && sub == 0) {
            fref[0] = root;
            fmeta[0] = (root >= 0) ? __float_as_int(aux[REF_ID(root)].w) : 0;
        }
        for (int it = 0; it < 40; ++it) {
            // ---- which slots expand, which are carried (leaves: budget 1) ----
            unsigned expm = 0, carm = 0;
#pragma unroll
            for (int j = 0; j < BK_HS; ++j) {
                const bool act = fref[j] != -1;
                const bool ex = act && (fref[j] < -1 || fmeta[j] < 0);
                expm |= (ex ? 1u : 0u) << j;
                carm |= ((act && !ex) ? 1u : 0u) << j;
            }
            // ---- children ----
            int cx[NC];                           // per child: hash slot -> column -> score bits
            unsigned vm = 0, spm = 0;             // children that exist; those that are spine nodes (already scored)
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int j = c >> 1, side = c & 1;
                int cref = -1;
                if ((expm >> j) & 1) {
                    cref = (fref[j] >= 0) ? fref[j] + ((~fmeta[j]) >> 4) + 1 + side       // same chunk: the height bits carry over
                                          : __float_as_int(sp.node[-fref[j] - 2][D + 4 + side]);
                    vm |= 1u << c;
                }
                place(cref, c, cx, spm);
            }
            if (!__syncthreads_or(expm != 0)) break;
            nv += __popc(vm);
            score_level(cx, vm, spm);
            // ---- rank the query's 32 children: (score desc, position asc); position = 8 sub + c ----
            float sc[NC];
            int rank[NC];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                sc[c] = ((vm >> c) & 1) ? __int_as_float(cx[c]) : FS_NEG_SCORE;
                rank[c] = 0;
            }
#pragma unroll
            for (int i = 0; i < NC; ++i)
#pragma unroll
                for (int k = i + 1; k < NC; ++k) {
                    const bool first = sc[i] >= sc[k];                  // i is the earlier position: it wins ties
                    rank[k] += first ? 1 : 0;
                    rank[i] += first ? 0 : 1;
                }
#pragma unroll 1
            for (int p = 1; p < BK_T; ++p) {
                // a partner's children come first on ties iff its slots are the lower ones: then "ahead of mine" is >=, which
                // for floats is > against the next value below mine
                const bool plow = (sub ^ p) < sub;
                float lim[NC];
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int bits = __float_as_int(sc[c]);
                    lim[c] = plow ? __int_as_float(sc[c] > 0.0f ? bits - 1 : (sc[c] < 0.0f ? bits + 1 : (int)0x80000001)) : sc[c];
                }
#pragma unroll
                for (int o = 0; o < NC; ++o) {
                    const float po = __shfl_xor_sync(FS_FULL, sc[o], p);
#pragma unroll
                    for (int c = 0; c < NC; ++c) rank[c] += (po > lim[c]) ? 1 : 0;
                }
            }
            unsigned car_all = carm << (BK_HS * sub);
            car_all |= __shfl_xor_sync(FS_FULL, car_all, 1);
            car_all |= __shfl_xor_sync(FS_FULL, car_all, 2);
            const int ncar = __popc(car_all);
            // ---- the new frontier through its shared-memory row: carried first in slot order, then the kept children ----
#pragma unroll
            for (int j = 0; j < BK_HS; ++j) { frs_ref[(BK_HS * sub + j) * 128] = -1; frs_meta[(BK_HS * sub + j) * 128] = 0; }
            __syncwarp();
            if (isq) {
#pragma unroll
                for (int j = 0; j < BK_HS; ++j) {
                    if ((carm >> j) & 1) {
                        const int pos = __popc(car_all & ((1u << (BK_HS * sub + j)) - 1u));
                        frs_ref[pos * 128] = fref[j]; frs_meta[pos * 128] = fmeta[j];
                    }
                }
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int j = c >> 1, side = c & 1;
                    if (((vm >> c) & 1) && sc[c] > 0.5f * FS_NEG_SCORE && ncar + rank[c] < W) {
                        const int cref = (fref[j] >= 0) ? fref[j] + ((~fmeta[j]) >> 4) + 1 + side
                                                        : __float_as_int(sp.node[-fref[j] - 2][D + 4 + side]);
                        const int pos = ncar + rank[c];
                        frs_ref[pos * 128] = cref;
                        frs_meta[pos * 128] = (cref >= 0) ? __float_as_int(aux[REF_ID(cref)].w) : 0;
                    }
                }
            }
            __syncwarp();
#pragma unroll
            for (int j = 0; j < BK_HS; ++j) { fref[j] = frs_ref[(BK_HS * sub + j) * 128]; fmeta[j] = frs_meta[(BK_HS * sub + j) * 128]; }
            __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < BK_HS; ++j)
            cells[f][j] = (isq && BK_HS * sub + j < width && fref[j] >= 0 && fmeta[j] >= 0) ? fmeta[j] : -1;
    }
    // ---- union (the second beam's repeats of a main cell blanked) and the hand-off to the block re-rank ----
    {
#pragma unroll 1
        for (int p = 0; p < BK_T; ++p) {
#pragma unroll
            for (int o = 0; o < BK_HS; ++o) {
                const int mc = __shfl_xor_sync(FS_FULL, cells[0][o], p);
#pragma unroll
                for (int j = 0; j < BK_HS; ++j)
                    if (cells[1][j] == mc) cells[1][j] = -1;
            }
        }
        int nv_q = nv + __shfl_xor_sync(FS_FULL, nv, 1);
        nv_q += __shfl_xor_sync(FS_FULL, nv_q, 2);
        if (qi < a.Bq) {
            const int64_t row = ((int64_t)t * gridDim.x + blk) * a.Bq + qi;     // (B,H,Npad) flattened
#pragma unroll
            for (int j = 0; j < BK_HS; ++j) {
                const int s = BK_HS * sub + j;
                if (s < a.width) a.cand[row * Wc + s] = cells[0][j];
                if (s < a.width2) a.cand[row * Wc + a.width + s] = cells[1][j];
            }
            if (a.nvis && sub == 0) a.nvis[row] = isq ? nv_q : 0;
        }
    }
}

template <int D>
cudaError_t launch_beam_block(const SelArgs& A, dim3 grid, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(fsb_beam_block_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BeamSmem<D>::TOTAL);
    if (e != cudaSuccess) return e;
    fsb_beam_block_kernel<D><<<grid, BK_THREADS, BeamSmem<D>::TOTAL, st>>>(A);
    return cudaSuccess;
}
