// ela_implicit.cuh -- auction on implicit low-rank costs C = Q K^T, cost
// tiles on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
// Included by ela_auction.cu (device part inside its anonymous namespace).
//
// The reference plans this as solve_implicit(Q, K, ...): "Load tiles of Q, K
// into SRAM; compute tile C_block = Q_block K_block^T using Tensor Cores; apply
// Auction update logic on registers/SRAM" (optimization_plan.md:11-22).  The
// cost matrix is never stored: one CTA per problem keeps the problem's K
// factor (M x D) in shared memory; each round gathers the bidding rows' Q rows
// (up to ELA_IMP_NB at a time) and computes their cost rows as
//   D[j, b] = sum_k K[j, k] * Q[i_b, k]      (A = K tile, 128 columns j of the
//                                             cost; B = the bidders' Q rows)
// with tcgen05.mma (kind::f16, bf16 or fp16 operands, fp32 accumulation), one
// 128-column tile of the cost per MMA.  TMEM lane j of a tile then holds
// column j's cost for every bidder, so warp w (TMEM lanes 32w..32w+31) reads
// 32 columns with tcgen05.ld and folds them into exact per-bidder top-2 states
// (ties included, as the explicit kernels do); a warp reduction and a merge of
// the warps' partials give each bidder's top-2 and bid.  The election is the
// one-CTA kernel's.
//
// Cost values: each element is the fp32 result of the same MMA instruction
// sequence (D/16 K-steps in order) whatever the round or bidder set, so a
// solve equals the explicit solve of the matrix this kernel materialises with
// the same instructions (ela_auction_implicit_costs); that matrix equals the
// fp32 product Q K^T up to fp32 rounding of the dot products.

#define ELA_IMP_THREADS 128   // one warpgroup: warp w reads TMEM lanes 32w..32w+31
#define ELA_IMP_NB 64         // bidders per MMA pass (the MMA's N dimension, padded to 16)
#define ELA_IMP_TMEM_COLS 256 // 4 column tiles x 64 bidders
#define ELA_IMP_MAX_TILES 4   // M <= 512

struct ImpParams {
    const void* Q;   // (B, N, D) bf16 / fp16, contiguous
    const void* Kf;  // (B, M, D), same dtype, contiguous
    int half;        // 1: fp16, 0: bf16
    int64_t B, N, M, D;
    double eps[ELA_MAX_PHASES];
    int n_eps, max_iter, tie_rule;
    int64_t* assign_out;
    float* prices_out;
    int64_t* stats_out;
    int32_t* status;
    float* cost_out;  // non-null: write the (B, N, M) costs and solve nothing
    unsigned long long wait_ns;
};

// Shared-memory layout of the implicit kernel (bytes).
struct ILayout {
    size_t ks, qs, P, win, owner, rowcol, act, lbid, lrow, lcol, wpart, total;
    int kc;  // row-cache entries per row (0: no cache)
    size_t ccol, ccost, ctau, ccnt, mrow, ment, scr;
};
#define ELA_IMP_KC 16          // row-cache entries per row
#define ELA_IMP_SCR 8          // bidder rows of costs staged in shared memory per cache build
#define ELA_IMP_SMEM_2CTA 115000  // dynamic shared memory that still lets two CTAs share an SM
__host__ __device__ inline ILayout i_layout(int64_t N, int64_t M, int64_t D) {
    ILayout L;
    const int64_t T = (M + 127) / 128;
    size_t o = 0;
    L.ks = o;     o = align_up(o + (size_t)(T * 128) * D * 2, 128);       // K factor, core-matrix layout
    L.qs = o;     o = align_up(o + (size_t)ELA_IMP_NB * D * 2, 128);      // the bidders' Q rows
    L.P = o;      o = align_up(o + 4 * (size_t)M, 16);
    L.win = o;    o = align_up(o + 4 * (size_t)M, 16);
    L.owner = o;  o = align_up(o + 4 * (size_t)M, 16);
    L.rowcol = o; o = align_up(o + 4 * (size_t)N, 16);
    L.act = o;    o = align_up(o + 4 * (size_t)N, 16);
    L.lbid = o;   o = align_up(o + 4 * (size_t)N, 16);
    L.lrow = o;   o = align_up(o + 4 * (size_t)N, 16);
    L.lcol = o;   o = align_up(o + 4 * (size_t)N, 16);
    L.wpart = o;  o = align_up(o + sizeof(Top2<float>) * 4 * ELA_IMP_NB, 16);
    L.total = o;
    // row cache (M a multiple of 128, at most 512 columns): kept only while
    // two CTAs still fit on an SM
    L.kc = 0;
    L.ccol = L.ccost = L.ctau = L.ccnt = L.mrow = L.ment = L.scr = 0;
    if (M % 128 == 0 && M <= 512) {
        const int kc = ELA_IMP_KC;
        L.ccol = o;  o = align_up(o + 2 * (size_t)N * kc, 16);  // cached columns
        L.ccost = o; o = align_up(o + 4 * (size_t)N * kc, 16);  // their costs
        L.ctau = o;  o = align_up(o + 4 * (size_t)N, 16);       // bound of every other column's value
        L.ccnt = o;  o = align_up(o + (size_t)N, 16);           // entries (0: none)
        L.mrow = o;  o = align_up(o + 4 * (size_t)N, 16);       // this round's cache misses: row,
        L.ment = o;  o = align_up(o + 4 * (size_t)N, 16);       //   and its bid entry
        L.scr = o;   o = align_up(o + 4 * (size_t)ELA_IMP_SCR * M, 16);  // staged cost rows
        if (o <= ELA_IMP_SMEM_2CTA) { L.kc = kc; L.total = o; }
    }
    return L;
}

// Cost rows staged in shared memory, read by the cache build's scan.
struct SharedRow {
    __device__ __forceinline__ uint4 load(const uint4* ptr) const { return *ptr; }
};

// 8 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __uint_as_float(r[k]);
}

// Cache build of one staged cost row (M = 128 * nch columns): exact top-2 and
// a new cache for the row.
__device__ __forceinline__ Top2<float> imp_build(int nch, const float* row, const float* P, int lane, int kc,
                                                 unsigned short* ccol, float* ccost, float* ctau, unsigned char* ccnt) {
    switch (nch) {
    case 1: return scan_build<float, 1, SharedRow>(row, P, lane, kc, ccol, ccost, ctau, ccnt, SharedRow());
    case 2: return scan_build<float, 2, SharedRow>(row, P, lane, kc, ccol, ccost, ctau, ccnt, SharedRow());
    case 3: return scan_build<float, 3, SharedRow>(row, P, lane, kc, ccol, ccost, ctau, ccnt, SharedRow());
    default: return scan_build<float, 4, SharedRow>(row, P, lane, kc, ccol, ccost, ctau, ccnt, SharedRow());
    }
}

// Byte offset of element (r, k) of a K-major operand tile with D columns in the
// tensor cores' no-swizzle canonical layout: 8-row x 16-byte core matrices,
// consecutive along K (LBO = 128 B), 8-row groups SBO = D/8 * 128 B apart.
__device__ __forceinline__ uint32_t core_off(int r, int k, int D) {
    return (uint32_t)((r >> 3) * (D >> 3) * 128 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

// Shared-memory matrix descriptor (no swizzle, K-major): start, LBO, SBO in
// 16-byte units, version 1 (bits 46-47).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// Instruction descriptor: fp32 accumulator, A and B bf16 (or fp16), both
// K-major, M = 128, N = n (multiple of 16).
__device__ __forceinline__ uint32_t umma_idesc(int n, int half) {
    const uint32_t ab = half ? 0u : 1u;
    return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int accum) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                 ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0), "r"(0), "r"(0), "r"(0)
                 : "memory");
}
__device__ __forceinline__ void tc_commit(unsigned long long* mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(mbar)) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 16 consecutive TMEM columns of this thread's lane (warp w: lanes 32w..).
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = __uint_as_float(r[k]);
}

// Costs of up to ELA_IMP_NB rows (rows[0..nb)) of problem b against all M
// columns into TMEM: gather the rows' Q into the B tile, one thread issues
// the MMAs (tiles x D/16 K-steps) and commits to the mbarrier, everyone waits.
// Returns false on a wait that ran past its limit.
__device__ bool imp_mma_pass(const ImpParams& p, const uint16_t* Qb, int nb, const int* rows, unsigned char* smem,
                             const ILayout& L, uint32_t tmem, unsigned long long* mbar, unsigned int& phase, int T,
                             int npad, const volatile int* abort) {
    const int D = (int)p.D, tid = threadIdx.x;
    // gather: 16-byte pieces (8 elements) of each row's D values; pad rows zero
    const int pieces = npad * (D >> 3);
    for (int x = tid; x < pieces; x += blockDim.x) {
        const int r = x / (D >> 3), kc = x % (D >> 3);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < nb) v = *reinterpret_cast<const uint4*>(Qb + (size_t)rows[r] * D + kc * 8);
        *reinterpret_cast<uint4*>(smem + L.qs + core_off(r, kc * 8, D)) = v;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the tensor cores read what threads wrote
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        tc_fence_after();
        const uint32_t idesc = umma_idesc(npad, p.half);
        const uint32_t sbo = (uint32_t)(D >> 3) * 128u;
        const uint32_t ks = smem_addr(smem + L.ks), qs = smem_addr(smem + L.qs);
        for (int t = 0; t < T; ++t)
            for (int s = 0; s < (D >> 4); ++s) {
                const uint64_t ad = umma_desc(ks + (uint32_t)t * 16u * sbo + (uint32_t)s * 256u, 128u, sbo);
                const uint64_t bd = umma_desc(qs + (uint32_t)s * 256u, 128u, sbo);
                tc_mma(tmem + (uint32_t)(t * ELA_IMP_NB), ad, bd, idesc, s > 0);
            }
        tc_commit(mbar);
    }
    __syncthreads();
    const bool ok = mbar_wait(mbar, phase, p.wait_ns, abort);
    phase ^= 1u;
    tc_fence_after();
    return __syncthreads_and(ok) != 0;
}

__global__ void __launch_bounds__(ELA_IMP_THREADS, 1) implicit_kernel(const ImpParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) unsigned long long s_mbar;
    __shared__ uint32_t s_tmem;
    __shared__ int s_nact, s_fail, s_nmiss;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = (int)p.N, M = (int)p.M, D = (int)p.D;
    const int T = (M + 127) / 128;
    const ILayout L = i_layout(N, M, D);
    float* P = reinterpret_cast<float*>(smem + L.P);
    unsigned int* Pbits = reinterpret_cast<unsigned int*>(smem + L.P);  // prices >= 0: bit order is value order
    int* win = reinterpret_cast<int*>(smem + L.win);
    int* owner = reinterpret_cast<int*>(smem + L.owner);
    int* rowcol = reinterpret_cast<int*>(smem + L.rowcol);
    int* act = reinterpret_cast<int*>(smem + L.act);
    float* lbid = reinterpret_cast<float*>(smem + L.lbid);
    int* lrow = reinterpret_cast<int*>(smem + L.lrow);
    int* lcol = reinterpret_cast<int*>(smem + L.lcol);
    Top2<float>* wpart = reinterpret_cast<Top2<float>*>(smem + L.wpart);
    const int kc = L.kc;
    unsigned short* ccol = reinterpret_cast<unsigned short*>(smem + L.ccol);
    float* ccost = reinterpret_cast<float*>(smem + L.ccost);
    float* ctau = reinterpret_cast<float*>(smem + L.ctau);
    unsigned char* ccnt = smem + L.ccnt;
    int* mrow = reinterpret_cast<int*>(smem + L.mrow);
    int* ment = reinterpret_cast<int*>(smem + L.ment);
    float* scr = reinterpret_cast<float*>(smem + L.scr);
    const float tol = 1e-5f;

    if (warp == 0) {  // TMEM columns for the accumulators, held until exit
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(&s_tmem)), "r"(ELA_IMP_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        s_fail = 0;  // (never set: the MMA waits only need a quiet abort flag)
        mbar_init(&s_mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    unsigned int phase = 0;
    bool failed = false;

    for (int64_t b = blockIdx.x; b < p.B && !failed; b += gridDim.x) {
        const uint16_t* Qb = reinterpret_cast<const uint16_t*>(p.Q) + (size_t)b * N * D;
        const uint16_t* Kb = reinterpret_cast<const uint16_t*>(p.Kf) + (size_t)b * M * D;
        // the K factor into shared memory (rows M..128T zero)
        for (int x = tid; x < T * 128 * (D >> 3); x += blockDim.x) {
            const int r = x / (D >> 3), kc = x % (D >> 3);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < M) v = *reinterpret_cast<const uint4*>(Kb + (size_t)r * D + kc * 8);
            *reinterpret_cast<uint4*>(smem + L.ks + core_off(r, kc * 8, D)) = v;
        }
        for (int j = tid; j < M; j += blockDim.x) { P[j] = 0.f; win[j] = 0; owner[j] = -1; }
        if (tid == 0) { s_nact = 0; s_nmiss = 0; }  // (both return to 0 in every round's election)
        for (int i = tid; i < N; i += blockDim.x) rowcol[i] = -1;
        if (kc > 0)
            for (int i = tid; i < N; i += blockDim.x) ccnt[i] = 0;
        __syncthreads();

        if (p.cost_out) {  // materialise the costs with the same MMA sequence
            for (int r0 = 0; r0 < N && !failed; r0 += ELA_IMP_NB) {
                const int nb = min(ELA_IMP_NB, N - r0);
                for (int x = tid; x < nb; x += blockDim.x) act[x] = r0 + x;
                __syncthreads();
                const int npad = (nb + 15) & ~15;
                if (!imp_mma_pass(p, Qb, nb, act, smem, L, tmem, &s_mbar, phase, T, npad, &s_fail)) { failed = true; break; }
                for (int t = 0; t < T; ++t)
                    for (int c0 = 0; c0 < npad; c0 += 16) {
                        float v[16];
                        tc_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(t * ELA_IMP_NB + c0), v);
                        const int j = t * 128 + 32 * warp + lane;
#pragma unroll
                        for (int k = 0; k < 16; ++k)
                            if (j < M && c0 + k < nb) p.cost_out[((size_t)b * N + r0 + c0 + k) * M + j] = v[k];
                    }
                tc_fence_before();
                __syncthreads();
            }
            continue;
        }

        long long rounds = 0, rowbids = 0;
        for (int ph = 0; ph < p.n_eps && !failed; ++ph) {
            const float eps = (float)p.eps[ph];
            for (int i = tid; i < N; i += blockDim.x) rowcol[i] = -1;
            for (int j = tid; j < M; j += blockDim.x) owner[j] = -1;
            __syncthreads();
            for (int it = 0; it < p.max_iter; ++it) {
                // ---- active rows (their order does not change the round)
                for (int i = tid; i < N; i += blockDim.x)
                    if (rowcol[i] < 0) act[atomicAdd(&s_nact, 1)] = i;
                __syncthreads();
                const int K = s_nact;
                if (K == 0) break;
                if (kc > 0) {
                    // ---- bids from the row caches (prices never fall, so a
                    //      cache whose second value is above its bound holds the
                    //      row's exact top-2); the misses go through the MMA
                    for (int k = warp; k < K; k += ELA_IMP_THREADS / 32) {
                        const int i = act[k], n = ccnt[i];
                        Top2<float> tt;
                        const bool hit = n >= 2 && cache_top2<float>(P, ccol + (size_t)i * kc, ccost + (size_t)i * kc,
                                                                      n, ctau[i], lane, tt);
                        if (lane == 0) {
                            if (hit) {
                                const int j1 = (tt.p2 >= 0 && !(tt.p1 == 0 && tt.p2 == 1)) ? tt.p2 : tt.p1;
                                lbid[k] = add_rn(P[j1], add_rn(sub_rn(tt.v1, tt.v2), eps));
                                lrow[k] = i;
                                lcol[k] = j1;
                            } else {
                                const int m = atomicAdd(&s_nmiss, 1);
                                mrow[m] = i;
                                ment[m] = k;
                            }
                        }
                    }
                    __syncthreads();
                    const int nm = s_nmiss;
                    for (int m0 = 0; m0 < nm; m0 += ELA_IMP_NB) {
                        const int nb = min(ELA_IMP_NB, nm - m0), npad = (nb + 15) & ~15;
                        if (!imp_mma_pass(p, Qb, nb, mrow + m0, smem, L, tmem, &s_mbar, phase, T, npad, &s_fail)) {
                            failed = true;
                            break;
                        }
                        for (int c0 = 0; c0 < nb; c0 += ELA_IMP_SCR) {
                            // stage ELA_IMP_SCR rows of costs (lane = column), then
                            // one warp per row: exact top-2, bid, new cache
                            for (int t = 0; t < T; ++t) {
                                float v[ELA_IMP_SCR];
                                tc_ld8(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(t * ELA_IMP_NB + c0), v);
                                const int j = t * 128 + 32 * warp + lane;
#pragma unroll
                                for (int k = 0; k < ELA_IMP_SCR; ++k) scr[k * M + j] = v[k];
                            }
                            __syncthreads();
                            for (int k = warp; k < ELA_IMP_SCR && c0 + k < nb; k += ELA_IMP_THREADS / 32) {
                                const int m = m0 + c0 + k, i = mrow[m], e = ment[m];
                                const Top2<float> tt = imp_build(T, scr + k * M, P, lane, kc, ccol + (size_t)i * kc,
                                                                 ccost + (size_t)i * kc, ctau + i, ccnt + i);
                                if (lane == 0) {
                                    const int j1 = (tt.p2 >= 0 && !(tt.p1 == 0 && tt.p2 == 1)) ? tt.p2 : tt.p1;
                                    lbid[e] = add_rn(P[j1], add_rn(sub_rn(tt.v1, tt.v2), eps));
                                    lrow[e] = i;
                                    lcol[e] = j1;
                                }
                            }
                            __syncthreads();  // the staged rows are read before the next ones land
                        }
                        tc_fence_before();
                        __syncthreads();
                    }
                }
                // ---- bids, ELA_IMP_NB rows per MMA pass (no row cache)
                for (int k0 = 0; k0 < K && kc == 0; k0 += ELA_IMP_NB) {
                    const int nb = min(ELA_IMP_NB, K - k0), npad = (nb + 15) & ~15;
                    if (!imp_mma_pass(p, Qb, nb, act + k0, smem, L, tmem, &s_mbar, phase, T, npad, &s_fail)) {
                        failed = true;
                        break;
                    }
                    for (int c0 = 0; c0 < npad; c0 += 16) {
                        Top2<float> st[16];
#pragma unroll
                        for (int k = 0; k < 16; ++k) top2_init(st[k]);
                        for (int t = 0; t < T; ++t) {  // this lane's columns in increasing order
                            float v[16];
                            tc_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(t * ELA_IMP_NB + c0), v);
                            const int j = t * 128 + 32 * warp + lane;
                            if (j < M) {
                                const float pj = P[j];
#pragma unroll
                                for (int k = 0; k < 16; ++k) top2_add(st[k], sub_rn(-v[k], pj), j);
                            }
                        }
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            if (c0 + k < nb) {  // padding slots of the MMA's N dimension need no reduction
                                const Top2<float> r = top2_warp(st[k]);
                                if (lane == 0) wpart[warp * ELA_IMP_NB + c0 + k] = r;
                            }
                        }
                    }
                    tc_fence_before();
                    __syncthreads();
                    for (int e = tid; e < nb; e += blockDim.x) {  // merge the 4 warps' partials: column, bid
                        Top2<float> r = wpart[e];
                        for (int w = 1; w < 4; ++w) r = top2_merge(r, wpart[w * ELA_IMP_NB + e]);
                        const int j1 = (r.p2 >= 0 && !(r.p1 == 0 && r.p2 == 1)) ? r.p2 : r.p1;
                        lbid[k0 + e] = add_rn(P[j1], add_rn(sub_rn(r.v1, r.v2), eps));
                        lrow[k0 + e] = act[k0 + e];
                        lcol[k0 + e] = j1;
                    }
                    __syncthreads();
                }
                if (failed) break;
                rounds++;
                rowbids += K;
                // ---- election: new price = max bid (in place: every bid is
                //      above its column's price); the largest key within 1e-5
                //      of it wins.  The round counters return to 0 here (all
                //      threads read them before this round's first barrier).
                for (int e = tid; e < K; e += blockDim.x) atomicMax(&Pbits[lcol[e]], __float_as_uint(lbid[e]));
                __syncthreads();
                for (int e = tid; e < K; e += blockDim.x) {
                    const int j = lcol[e];
                    if (absval(sub_rn(lbid[e], P[j])) < tol) atomicMax(&win[j], win_key(lrow[e], N, p.tie_rule));
                }
                __syncthreads();
                for (int e = tid; e < K; e += blockDim.x) {
                    const int j = lcol[e], i = lrow[e];
                    if (win[j] == win_key(i, N, p.tie_rule)) {
                        const int prev = owner[j];
                        if (prev >= 0) rowcol[prev] = -1;
                        owner[j] = i;
                        rowcol[i] = j;
                    }
                }
                if (tid == 0) { s_nact = 0; s_nmiss = 0; }
                __syncthreads();
                // win[] cleared before the next round's first barrier, which
                // every thread passes only after its share of this loop
                for (int e = tid; e < K; e += blockDim.x) win[lcol[e]] = 0;
            }
        }
        if (failed) break;
        int un = 0;
        for (int i = tid; i < N; i += blockDim.x) {
            p.assign_out[b * N + i] = rowcol[i];
            un += rowcol[i] < 0;
        }
        for (int j = tid; j < M; j += blockDim.x) p.prices_out[b * M + j] = P[j];
        if (tid == 0) s_nact = 0;
        __syncthreads();
        if (un) atomicAdd(&s_nact, un);
        __syncthreads();
        if (tid == 0 && p.stats_out) {
            p.stats_out[4 * b + 0] = rounds;
            p.stats_out[4 * b + 1] = rowbids;
            p.stats_out[4 * b + 2] = 0;
            p.stats_out[4 * b + 3] = s_nact;
        }
        __syncthreads();
    }
    if (failed && tid == 0) atomicCAS(p.status, ELA_OK, ELA_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ELA_IMP_TMEM_COLS) : "memory");
}
