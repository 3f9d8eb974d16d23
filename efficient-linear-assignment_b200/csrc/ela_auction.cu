// ela_auction.cu -- B200 (sm_100a) auction solver for the linear assignment problem.
//
// Device implementation of the Jacobi auction of the reference torch backend
// (src/efficient_linear_assignment/auction/torch_backend.py:9-159), with every
// round on the device and results identical to that backend run on one CPU
// thread:
//   values  v[j] = (-c[i][j]) - P[j]                           torch_backend.py:24,76
//   top-2   (v1, j1), v2 as torch.topk(k=2) returns them on CPU, ties included :81
//   bid     P[j1] + ((v1 - v2) + eps)                            :88,99
//   price   P[j] = max bid on j (bids never fall below P[j])     :102
//   winner  highest row whose |bid - P[j]| < 1e-5                :106-136
//   owner   the previous owner of a won column becomes unassigned :144-156
//
// Two kernels:
//   auction_cta_kernel   one CTA per problem, all state in shared memory,
//                        __syncthreads between the phases of a round.
//   auction_grid_kernel  S CTAs per problem (cooperative launch), one bounded
//                        barrier per round; the election is settled without a
//                        second barrier by linking every round's bidders on a
//                        column into a per-column list that each bidder walks
//                        after the barrier.
// The C ABI is declared in include/ela_auction.h.

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include "ela_auction.h"

#define ELA_MAX_PHASES 32
#define ELA_CTA_THREADS 512
#define ELA_GRID_THREADS 512
#define ELA_SMALL_M 128           // below this torch.topk uses introselect
#define ELA_ROWS_PER_CTA_MAX 8192 // owned-row state of the grid path lives in smem

namespace {

// ---------------------------------------------------------------- arithmetic
// Round-to-nearest operations spelled out so that no contraction or
// reassociation can change a result relative to the CPU reference.
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float absval(float a) { return fabsf(a); }
__device__ __forceinline__ double absval(double a) { return fabs(a); }

// Positive prices and bids order like their bit patterns, so the column max is
// an unsigned atomicMax on the bits; 0 means "no bid".
template <typename R> struct Bits;
template <> struct Bits<float> {
    typedef unsigned int U;
    static __device__ __forceinline__ U to(float x) { return __float_as_uint(x); }
    static __device__ __forceinline__ float from(U u) { return __uint_as_float(u); }
};
template <> struct Bits<double> {
    typedef unsigned long long U;
    static __device__ __forceinline__ U to(double x) { return (U)__double_as_longlong(x); }
    static __device__ __forceinline__ double from(U u) { return __longlong_as_double((long long)u); }
};

// ------------------------------------------------------------- cost loading
template <typename In> struct Elem;
template <> struct Elem<float> {
    static constexpr int W = 4;
    template <typename R> static __device__ __forceinline__ void unpack(const uint4& q, R* o) {
        o[0] = (R)__uint_as_float(q.x); o[1] = (R)__uint_as_float(q.y);
        o[2] = (R)__uint_as_float(q.z); o[3] = (R)__uint_as_float(q.w);
    }
    template <typename R> static __device__ __forceinline__ R one(const float* p) { return (R)__ldg(p); }
};
template <> struct Elem<__half> {
    static constexpr int W = 8;
    template <typename R> static __device__ __forceinline__ void unpack(const uint4& q, R* o) {
        const unsigned int w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            __half_raw lo, hi;
            lo.x = (unsigned short)(w[k] & 0xffffu);
            hi.x = (unsigned short)(w[k] >> 16);
            o[2 * k] = (R)__half2float(__half(lo));
            o[2 * k + 1] = (R)__half2float(__half(hi));
        }
    }
    template <typename R> static __device__ __forceinline__ R one(const __half* p) {
        __half_raw r; r.x = __ldg(reinterpret_cast<const unsigned short*>(p));
        return (R)__half2float(__half(r));
    }
};
template <> struct Elem<__nv_bfloat16> {
    static constexpr int W = 8;
    template <typename R> static __device__ __forceinline__ void unpack(const uint4& q, R* o) {
        const unsigned int w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            // bf16 -> fp32 is exact: the 16 bits are the top half of the float
            o[2 * k] = (R)__uint_as_float(w[k] << 16);
            o[2 * k + 1] = (R)__uint_as_float(w[k] & 0xffff0000u);
        }
    }
    template <typename R> static __device__ __forceinline__ R one(const __nv_bfloat16* p) {
        unsigned short h = __ldg(reinterpret_cast<const unsigned short*>(p));
        return (R)__uint_as_float(((unsigned int)h) << 16);
    }
};
template <> struct Elem<double> {
    static constexpr int W = 2;
    template <typename R> static __device__ __forceinline__ void unpack(const uint4& q, R* o) {
        o[0] = (R)__longlong_as_double((long long)(((unsigned long long)q.y << 32) | q.x));
        o[1] = (R)__longlong_as_double((long long)(((unsigned long long)q.w << 32) | q.z));
    }
    template <typename R> static __device__ __forceinline__ R one(const double* p) { return (R)__ldg(p); }
};

// 16-byte streaming load through the read-only path; the cost matrix is never
// written during a solve.
__device__ __forceinline__ uint4 ld_stream16(const void* ptr) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(ptr));
    return r;
}

// ------------------------------------------------------------------- top-2
// Running top-2 over one lane's columns (visited in increasing order) plus the
// first two columns that hold the maximum, which is what decides the column
// torch.topk reports when the maximum is tied.
template <typename R> struct Top2 {
    R v1, v2;
    int p1, p2;  // p1 < 0: empty; p2 < 0: maximum seen once
};

template <typename R> __device__ __forceinline__ void top2_init(Top2<R>& t) {
    t.v1 = -INFINITY; t.v2 = -INFINITY; t.p1 = -1; t.p2 = -1;
}

template <typename R> __device__ __forceinline__ void top2_add(Top2<R>& t, R v, int col) {
    if (t.p1 < 0 || v > t.v1) {
        t.v2 = t.v1; t.v1 = v; t.p1 = col; t.p2 = -1;
    } else if (v == t.v1) {
        if (t.p2 < 0) t.p2 = col;
        t.v2 = v;
    } else if (v > t.v2) {
        t.v2 = v;
    }
}

// Merge two disjoint column sets; commutative, so a butterfly leaves every
// lane with the same result.
template <typename R> __device__ __forceinline__ Top2<R> top2_merge(Top2<R> a, Top2<R> b) {
    if (a.p1 < 0) return b;
    if (b.p1 < 0) return a;
    if (a.v1 > b.v1) { a.v2 = (a.v2 > b.v1) ? a.v2 : b.v1; return a; }
    if (b.v1 > a.v1) { b.v2 = (b.v2 > a.v1) ? b.v2 : a.v1; return b; }
    Top2<R> r;
    r.v1 = a.v1; r.v2 = a.v1;
    const int big = 0x7fffffff;
    if (a.p1 < b.p1) {
        r.p1 = a.p1;
        const int ap2 = a.p2 >= 0 ? a.p2 : big;
        r.p2 = ap2 < b.p1 ? ap2 : b.p1;
    } else {
        r.p1 = b.p1;
        const int bp2 = b.p2 >= 0 ? b.p2 : big;
        r.p2 = bp2 < a.p1 ? bp2 : a.p1;
    }
    return r;
}

template <typename R> __device__ __forceinline__ Top2<R> top2_warp(Top2<R> t) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        Top2<R> o;
        o.v1 = __shfl_xor_sync(0xffffffffu, t.v1, off);
        o.v2 = __shfl_xor_sync(0xffffffffu, t.v2, off);
        o.p1 = __shfl_xor_sync(0xffffffffu, t.p1, off);
        o.p2 = __shfl_xor_sync(0xffffffffu, t.p2, off);
        t = top2_merge(t, o);
    }
    return t;
}

// ------------------------------------------------- small-row tie resolution
// For M < 128 torch.topk runs std::nth_element (introselect) on (value, index)
// pairs with less(a, b) := a.value > b.value and reports the pair left at
// position 0.  Only a tied maximum makes that choice matter; then one lane
// replays the introselect steps on the warp's copy of the row in shared memory.
template <typename R> struct PairRef {
    R* v;
    int* ix;
    __device__ __forceinline__ bool less(int a, int b) const { return v[a] > v[b]; }
    __device__ __forceinline__ void swap(int a, int b) const {
        R tv = v[a]; v[a] = v[b]; v[b] = tv;
        int ti = ix[a]; ix[a] = ix[b]; ix[b] = ti;
    }
};

// Heap helpers used only when the introselect depth budget runs out.
template <typename R>
__device__ void heap_push(const PairRef<R>& q, int hole, int top, R val, int vix) {
    int parent = (hole - 1) / 2;
    while (hole > top && q.v[parent] > val) {
        q.v[hole] = q.v[parent]; q.ix[hole] = q.ix[parent];
        hole = parent; parent = (hole - 1) / 2;
    }
    q.v[hole] = val; q.ix[hole] = vix;
}
template <typename R>
__device__ void heap_adjust(const PairRef<R>& q, int hole, int len, R val, int vix) {
    const int top = hole;
    int child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (q.less(child, child - 1)) child--;
        q.v[hole] = q.v[child]; q.ix[hole] = q.ix[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        q.v[hole] = q.v[child - 1]; q.ix[hole] = q.ix[child - 1];
        hole = child - 1;
    }
    heap_push(q, hole, top, val, vix);
}
template <typename R> __device__ void heap_select(PairRef<R> q, int len, int n) {
    if (len >= 2)
        for (int parent = (len - 2) / 2;; --parent) {
            heap_adjust(q, parent, len, q.v[parent], q.ix[parent]);
            if (parent == 0) break;
        }
    for (int i = len; i < n; ++i)
        if (q.less(i, 0)) {
            R val = q.v[i]; int vix = q.ix[i];
            q.v[i] = q.v[0]; q.ix[i] = q.ix[0];
            heap_adjust(q, 0, len, val, vix);
        }
}

// Returns the column torch.topk(k=2) reports first for v[0..n), n < 128.
template <typename R> __device__ int introselect_top1(R* v, int* ix, int n) {
    PairRef<R> q{v, ix};
    int first = 0, last = n;
    const int nth = 1;
    int lg = 0;
    while ((1 << (lg + 1)) <= n) lg++;
    int depth = 2 * lg;
    while (last - first > 3) {
        if (depth == 0) {
            PairRef<R> sub{v + first, ix + first};
            heap_select(sub, nth + 1 - first, last - first);
            q.swap(first, nth);
            return ix[0];
        }
        --depth;
        const int mid = first + (last - first) / 2, a = first + 1, b = mid, c = last - 1;
        int s;
        if (q.less(a, b)) {
            if (q.less(b, c)) s = b;
            else if (q.less(a, c)) s = c;
            else s = a;
        } else if (q.less(a, c)) s = a;
        else if (q.less(b, c)) s = c;
        else s = b;
        q.swap(first, s);
        int lo = first + 1, hi = last;
        for (;;) {
            while (q.less(lo, first)) ++lo;
            --hi;
            while (q.less(first, hi)) --hi;
            if (!(lo < hi)) break;
            q.swap(lo, hi);
            ++lo;
        }
        if (lo <= nth) first = lo; else last = lo;
    }
    for (int i = first + 1; i < last; ++i) {
        R val = v[i]; int vix = ix[i];
        if (val > v[first]) {
            for (int k = i; k > first; --k) { v[k] = v[k - 1]; ix[k] = ix[k - 1]; }
            v[first] = val; ix[first] = vix;
        } else {
            int k = i;
            while (val > v[k - 1]) { v[k] = v[k - 1]; ix[k] = ix[k - 1]; --k; }
            v[k] = val; ix[k] = vix;
        }
    }
    return ix[0];
}

// ------------------------------------------------------------------ params
struct Params {
    const void* cost;
    int64_t B, N, M, stride_b, stride_n;
    double eps[ELA_MAX_PHASES];
    int n_eps;
    int max_iter;
    int vec_ok;              // 16-byte vector loads are legal for every row
    int64_t* assign_out;
    void* prices_out;
    int64_t* stats_out;      // may be null
    int32_t* status;         // never null (points into the workspace if the caller passed none)
    unsigned char* ws;       // grid path workspace
    size_t group_bytes;      // grid path: workspace bytes per group
    int S;                   // grid path: CTAs per problem
    int ngroups;             // grid path: problems solved at once
    int rows_per_cta;        // grid path: ceil(N / S)
    unsigned long long wait_ns;
    int skip_arrive;
};

// --------------------------------------------------------------- one bid
// The warp computes one row's bid.  Every lane returns the same (j1, bid).
// scr_v / scr_i: this warp's 128-entry scratch, used only when M < 128.
template <typename In, typename R, int UNROLL>
__device__ __forceinline__ void bid_row(const Params& p, const In* row, const R* __restrict__ Ps,
                                        R eps, int lane, R* scr_v, int* scr_i, int& j1_out,
                                        R& bid_out) {
    const int M = (int)p.M;
    Top2<R> t;
    top2_init(t);
    if (p.vec_ok) {
        constexpr int W = Elem<In>::W;
        const int nchunks = M / W;
        const uint4* rv = reinterpret_cast<const uint4*>(row);
        for (int base = 0; base < nchunks; base += 32 * UNROLL) {
            uint4 raw[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const int ch = base + 32 * u + lane;
                if (ch < nchunks) raw[u] = ld_stream16(rv + ch);
            }
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const int ch = base + 32 * u + lane;
                if (ch < nchunks) {
                    R x[W];
                    Elem<In>::template unpack<R>(raw[u], x);
#pragma unroll
                    for (int e = 0; e < W; ++e) {
                        const int col = ch * W + e;
                        top2_add(t, sub_rn(-x[e], Ps[col]), col);
                    }
                }
            }
        }
    } else {
        for (int col = lane; col < M; col += 32)
            top2_add(t, sub_rn(-Elem<In>::template one<R>(row + col), Ps[col]), col);
    }
    t = top2_warp(t);
    int j1;
    if (t.v1 == t.v2 && M < ELA_SMALL_M) {
        for (int col = lane; col < M; col += 32) {
            scr_v[col] = sub_rn(-Elem<In>::template one<R>(row + col), Ps[col]);
            scr_i[col] = col;
        }
        __syncwarp();
        int r = 0;
        if (lane == 0) r = introselect_top1<R>(scr_v, scr_i, M);
        j1 = __shfl_sync(0xffffffffu, r, 0);
        __syncwarp();
    } else {
        j1 = (t.p2 >= 0 && !(t.p1 == 0 && t.p2 == 1)) ? t.p2 : t.p1;
    }
    j1_out = j1;
    bid_out = add_rn(Ps[j1], add_rn(sub_rn(t.v1, t.v2), eps));
}

// ======================================================= one CTA per problem
// Shared-memory layout (byte offsets), identical on host and device.
struct CtaLayout {
    size_t win, P, bidval, MB, owner, assign, bidcol, active, scr_v, scr_i, total;
};
__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

template <typename R>
__host__ __device__ inline CtaLayout cta_layout(int64_t N, int64_t M, int warps) {
    typedef typename std::conditional<sizeof(R) == 4, unsigned int, unsigned long long>::type U;
    CtaLayout L;
    size_t o = 0;
    L.win = o;    o = align_up(o + 8 * (size_t)M, 16);
    L.P = o;      o = align_up(o + sizeof(R) * (size_t)M, 16);
    L.bidval = o; o = align_up(o + sizeof(R) * (size_t)N, 16);
    L.MB = o;     o = align_up(o + sizeof(U) * (size_t)M, 16);
    L.owner = o;  o = align_up(o + 4 * (size_t)M, 16);
    L.assign = o; o = align_up(o + 4 * (size_t)N, 16);
    L.bidcol = o; o = align_up(o + 4 * (size_t)N, 16);
    L.active = o; o = align_up(o + 4 * (size_t)N, 16);
    const size_t scr = (M < ELA_SMALL_M) ? (size_t)warps * ELA_SMALL_M : 0;
    L.scr_v = o;  o = align_up(o + sizeof(R) * scr, 16);
    L.scr_i = o;  o = align_up(o + 4 * scr, 16);
    L.total = o;
    return L;
}

template <typename In, typename R>
__global__ void __launch_bounds__(ELA_CTA_THREADS)
auction_cta_kernel(const Params p) {
    typedef Bits<R> BT;
    typedef typename BT::U U;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_nact;
    __shared__ int s_unassigned;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int N = (int)p.N, M = (int)p.M;
    const CtaLayout L = cta_layout<R>(N, M, nw);
    unsigned long long* win = reinterpret_cast<unsigned long long*>(smem + L.win);
    R* P = reinterpret_cast<R*>(smem + L.P);
    R* bidval = reinterpret_cast<R*>(smem + L.bidval);
    U* MB = reinterpret_cast<U*>(smem + L.MB);
    int* owner = reinterpret_cast<int*>(smem + L.owner);
    int* assign = reinterpret_cast<int*>(smem + L.assign);
    int* bidcol = reinterpret_cast<int*>(smem + L.bidcol);
    int* active = reinterpret_cast<int*>(smem + L.active);
    R* scr_v = reinterpret_cast<R*>(smem + L.scr_v) + warp * ELA_SMALL_M;
    int* scr_i = reinterpret_cast<int*>(smem + L.scr_i) + warp * ELA_SMALL_M;
    const R tol = (R)1e-5;

    for (int64_t b = blockIdx.x; b < p.B; b += gridDim.x) {
        const In* base = reinterpret_cast<const In*>(p.cost) + b * p.stride_b;
        for (int j = tid; j < M; j += blockDim.x) { P[j] = (R)0; MB[j] = 0; win[j] = 0ull; }
        long long rounds = 0, rowbids = 0;
        unsigned int tag = 0;
        for (int ph = 0; ph < p.n_eps; ++ph) {
            const R eps = (R)p.eps[ph];
            for (int j = tid; j < M; j += blockDim.x) owner[j] = -1;
            for (int i = tid; i < N; i += blockDim.x) assign[i] = -1;
            __syncthreads();
            for (int it = 0; it < p.max_iter; ++it) {
                // 1. active rows (order does not matter: the election below is
                //    by row id, and each row's bid depends only on its own row)
                if (tid == 0) s_nact = 0;
                __syncthreads();
                for (int i = tid; i < N; i += blockDim.x)
                    if (assign[i] < 0) active[atomicAdd(&s_nact, 1)] = i;
                __syncthreads();
                const int K = s_nact;
                if (K == 0) break;
                rounds++;
                rowbids += K;
                ++tag;
                // 2. bids against the round-start prices; column max of the bids
                for (int k = warp; k < K; k += nw) {
                    int j1;
                    R bid;
                    bid_row<In, R, 4>(p, base + (int64_t)active[k] * p.stride_n, P, eps, lane,
                                      scr_v, scr_i, j1, bid);
                    if (lane == 0) {
                        bidcol[k] = j1;
                        bidval[k] = bid;
                        atomicMax(&MB[j1], BT::to(bid));
                    }
                }
                __syncthreads();
                // 3. election: highest row within 1e-5 of the new price
                for (int k = tid; k < K; k += blockDim.x) {
                    const int j = bidcol[k];
                    if (absval(sub_rn(bidval[k], BT::from(MB[j]))) < tol)
                        atomicMax(&win[j], ((unsigned long long)tag << 32) | (unsigned int)active[k]);
                }
                __syncthreads();
                // 4. winners take their columns; previous owners drop out
                for (int k = tid; k < K; k += blockDim.x) {
                    const int j = bidcol[k], i = active[k];
                    if (win[j] == (((unsigned long long)tag << 32) | (unsigned int)i)) {
                        const int prev = owner[j];
                        if (prev >= 0) assign[prev] = -1;
                        owner[j] = i;
                        assign[i] = j;
                        P[j] = BT::from(MB[j]);
                        MB[j] = 0;
                    }
                }
                __syncthreads();
            }
        }
        // outputs
        if (tid == 0) s_unassigned = 0;
        __syncthreads();
        int mine = 0;
        for (int i = tid; i < N; i += blockDim.x) {
            const int a = assign[i];
            p.assign_out[b * p.N + i] = a;
            mine += (a < 0);
        }
        if (mine) atomicAdd(&s_unassigned, mine);
        R* pout = reinterpret_cast<R*>(p.prices_out) + b * p.M;
        for (int j = tid; j < M; j += blockDim.x) pout[j] = P[j];
        __syncthreads();
        if (tid == 0 && p.stats_out) {
            p.stats_out[4 * b + 0] = rounds;
            p.stats_out[4 * b + 1] = rowbids;
            p.stats_out[4 * b + 2] = 0;
            p.stats_out[4 * b + 3] = s_unassigned;
        }
        __syncthreads();
    }
}

// ================================================== S CTAs per problem (grid)
// Per-group workspace (global memory), byte offsets from the group base:
//   ctrl   [256]     bar (u32) at 0, cnt[3] (u32) at 128
//   MB     [3][M]    column max bid of a round, bits (0 = no bid); round t uses t%3
//   head   [2][M]    u64 (t+1)<<32 | row: last bidder linked on the column in round t
//   nbid   [2][N]    bid of row i in round t (parity t&1)
//   nnext  [2][N]    next bidder on the same column in round t, -1 = end
// A round's buffers are written in round t, read in round t+1 and rewritten
// no earlier than round t+2 (t+3 for MB/cnt, which are zeroed in round t+2),
// so a CTA that runs ahead never overwrites data a slower CTA still reads.
struct GroupLayout {
    size_t ctrl, MB, head, nbid, nnext, total;
};
template <typename R> __host__ __device__ inline GroupLayout group_layout(int64_t N, int64_t M) {
    GroupLayout L;
    size_t o = 0;
    L.ctrl = o;  o += 256;
    L.MB = o;    o = align_up(o + 3 * sizeof(R) * (size_t)M, 256);
    L.head = o;  o = align_up(o + 2 * 8 * (size_t)M, 256);
    L.nbid = o;  o = align_up(o + 2 * sizeof(R) * (size_t)N, 256);
    L.nnext = o; o = align_up(o + 2 * 4 * (size_t)N, 256);
    L.total = o;
    return L;
}
// workspace = [256 B launch control: abort flag, status] + ngroups * group bytes
#define ELA_WS_HEADER 256

struct GridSmem {
    size_t P, rowcol, rowbid, active, scr_v, scr_i, total;
};
template <typename R> __host__ __device__ inline GridSmem grid_smem(int64_t M, int rpc, int warps) {
    GridSmem L;
    size_t o = 0;
    L.P = o;      o = align_up(o + sizeof(R) * (size_t)M, 16);
    L.rowcol = o; o = align_up(o + 4 * (size_t)rpc, 16);
    L.rowbid = o; o = align_up(o + 4 * (size_t)rpc, 16);
    L.active = o; o = align_up(o + 4 * (size_t)rpc, 16);
    const size_t scr = (M < ELA_SMALL_M) ? (size_t)warps * ELA_SMALL_M : 0;
    L.scr_v = o;  o = align_up(o + sizeof(R) * scr, 16);
    L.scr_i = o;  o = align_up(o + 4 * scr, 16);
    L.total = o;
    return L;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned int* p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Barrier of the S CTAs of one group.  The counter only grows; CTA c waits
// until it reaches `target` (S more per round).  Every wait is bounded: past
// p.wait_ns the waiter raises the launch-wide abort flag and records
// ELA_ERR_TIMEOUT; any waiter that sees the flag gives up too.  Returns false
// when the caller must leave the kernel.
__device__ __forceinline__ bool group_barrier(const Params& p, unsigned int* bar, unsigned int target,
                                              int* abort_flag, bool skip_arrive) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        __threadfence();
        if (!skip_arrive) red_release_add(bar, 1u);
        const unsigned long long t0 = globaltimer_ns();
        unsigned int spins = 0;
        for (;;) {
            const unsigned int v = ld_acquire_u32(bar);
            if ((int)(v - target) >= 0) break;
            if ((++spins & 63u) == 0) {
                if (*(volatile int*)abort_flag) { ok = 0; break; }
                if (globaltimer_ns() - t0 > p.wait_ns) {
                    atomicExch(abort_flag, 1);
                    atomicCAS(p.status, ELA_OK, ELA_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

template <typename In, typename R>
__global__ void __launch_bounds__(ELA_GRID_THREADS, 1)
auction_grid_kernel(const Params p) {
    typedef Bits<R> BT;
    typedef typename BT::U U;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_nact, s_unassigned;
    __shared__ unsigned int s_kprev;
    __shared__ int s_err;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int S = p.S, g = blockIdx.x / S, c = blockIdx.x % S;
    if (g >= p.ngroups) return;
    const int N = (int)p.N, M = (int)p.M, rpc = p.rows_per_cta;
    const int my_rows = (c < N) ? (N - 1 - c) / S + 1 : 0;  // rows c, c+S, c+2S, ...

    const GridSmem SL = grid_smem<R>(M, rpc, nw);
    R* Ps = reinterpret_cast<R*>(smem + SL.P);
    int* rowcol = reinterpret_cast<int*>(smem + SL.rowcol);  // assigned column or -1
    int* rowbid = reinterpret_cast<int*>(smem + SL.rowbid);  // column bid on last round or -1
    int* active = reinterpret_cast<int*>(smem + SL.active);
    R* scr_v = reinterpret_cast<R*>(smem + SL.scr_v) + warp * ELA_SMALL_M;
    int* scr_i = reinterpret_cast<int*>(smem + SL.scr_i) + warp * ELA_SMALL_M;

    int* abort_flag = reinterpret_cast<int*>(p.ws);
    const GroupLayout GL = group_layout<R>(N, M);
    unsigned char* gb = p.ws + ELA_WS_HEADER + (size_t)g * p.group_bytes;
    unsigned int* bar = reinterpret_cast<unsigned int*>(gb + GL.ctrl);
    unsigned int* cnt = reinterpret_cast<unsigned int*>(gb + GL.ctrl + 128);
    U* MBa = reinterpret_cast<U*>(gb + GL.MB);
    unsigned long long* heada = reinterpret_cast<unsigned long long*>(gb + GL.head);
    R* nbida = reinterpret_cast<R*>(gb + GL.nbid);
    int* nnexta = reinterpret_cast<int*>(gb + GL.nnext);
    const R tol = (R)1e-5;

    unsigned int t = 0;        // round tag, identical in all CTAs of the group
    unsigned int target = 0;   // barrier target
    bool first_barrier = true;
    if (tid == 0) s_err = 0;

    for (int64_t b = g; b < p.B; b += p.ngroups) {
        const In* base = reinterpret_cast<const In*>(p.cost) + b * p.stride_b;
        for (int j = tid; j < M; j += blockDim.x) Ps[j] = (R)0;
        for (int q = tid; q < my_rows; q += blockDim.x) { rowcol[q] = -1; rowbid[q] = -1; }
        long long rounds = 0, rowbids = 0;
        int ph = 0, it = 0;
        bool first = true;
        __syncthreads();
        if (p.max_iter > 0) {
            for (;;) {
                if (!first) {
                    // ---- apply round t-1: elections, evictions, prices
                    const unsigned int tp = t - 1;
                    const U* MBp = MBa + (size_t)(tp % 3) * M;
                    const unsigned long long* headp = heada + (size_t)(tp & 1) * M;
                    const R* nbidp = nbida + (size_t)(tp & 1) * N;
                    const int* nnextp = nnexta + (size_t)(tp & 1) * N;
                    for (int q = tid; q < my_rows; q += blockDim.x) {
                        const int i = c + q * S;
                        const int jb = rowbid[q];
                        if (jb >= 0) {
                            rowbid[q] = -1;
                            const unsigned long long h = __ldcg(headp + jb);
                            const R mb = BT::from(__ldcg(MBp + jb));
                            if ((unsigned int)(h >> 32) != t) { s_err = ELA_ERR_INTERNAL; continue; }
                            int cur = (int)(unsigned int)(h & 0xffffffffull), best = -1, steps = 0;
                            while (cur >= 0 && cur < N && steps <= N) {
                                const R bc = __ldcg(nbidp + cur);
                                const int nx = __ldcg(nnextp + cur);
                                if (cur > best && absval(sub_rn(bc, mb)) < tol) best = cur;
                                cur = nx;
                                ++steps;
                            }
                            if (steps > N || cur >= N) s_err = ELA_ERR_INTERNAL;
                            if (best == i) rowcol[q] = jb;
                        } else {
                            const int j = rowcol[q];
                            if (j >= 0 && (unsigned int)(__ldcg(headp + j) >> 32) == t) rowcol[q] = -1;
                        }
                    }
                    for (int j = tid; j < M; j += blockDim.x) {
                        const U u = __ldcg(MBp + j);
                        if (u) Ps[j] = BT::from(u);
                    }
                    if (tid == 0) s_kprev = __ldcg(cnt + (tp % 3));
                    __syncthreads();
                    const unsigned int kprev = s_kprev;
                    if (kprev > 0) { rounds++; rowbids += kprev; }
                    if (kprev == 0 || it == p.max_iter) {
                        if (++ph == p.n_eps) break;
                        it = 0;
                        for (int q = tid; q < my_rows; q += blockDim.x) rowcol[q] = -1;
                    }
                }
                first = false;
                const R eps = (R)p.eps[ph];
                // ---- zero round t+1's column maxima and counter
                {
                    U* MBn = MBa + (size_t)((t + 1) % 3) * M;
                    for (int j = c * blockDim.x + tid; j < M; j += S * blockDim.x) MBn[j] = 0;
                    if (c == 0 && tid == 0) cnt[(t + 1) % 3] = 0u;
                }
                // ---- bid
                if (tid == 0) s_nact = 0;
                __syncthreads();
                for (int q = tid; q < my_rows; q += blockDim.x)
                    if (rowcol[q] < 0) active[atomicAdd(&s_nact, 1)] = q;
                __syncthreads();
                const int K = s_nact;
                U* MBc = MBa + (size_t)(t % 3) * M;
                unsigned long long* headc = heada + (size_t)(t & 1) * M;
                R* nbidc = nbida + (size_t)(t & 1) * N;
                int* nnextc = nnexta + (size_t)(t & 1) * N;
                for (int k = warp; k < K; k += nw) {
                    const int q = active[k];
                    const int i = c + q * S;
                    int j1;
                    R bid;
                    bid_row<In, R, 8>(p, base + (int64_t)i * p.stride_n, Ps, eps, lane, scr_v, scr_i, j1, bid);
                    if (lane == 0) {
                        atomicMax(MBc + j1, BT::to(bid));
                        const unsigned long long old =
                            atomicExch(headc + j1, ((unsigned long long)(t + 1) << 32) | (unsigned int)i);
                        const int nx = ((unsigned int)(old >> 32) == t + 1) ? (int)(unsigned int)(old & 0xffffffffull) : -1;
                        __stcg(nbidc + i, bid);
                        __stcg(nnextc + i, nx);
                        rowbid[q] = j1;
                    }
                }
                if (tid == 0 && K > 0) atomicAdd(cnt + (t % 3), (unsigned int)K);
                ++it;
                target += S;
                const bool skip = p.skip_arrive && first_barrier && c == 0;
                first_barrier = false;
                if (!group_barrier(p, bar, target, abort_flag, skip)) return;
                ++t;
            }
        }
        // ---- outputs of problem b
        if (tid == 0) s_unassigned = 0;
        __syncthreads();
        int mine = 0;
        for (int q = tid; q < my_rows; q += blockDim.x) {
            const int a = rowcol[q];
            p.assign_out[b * p.N + c + (int64_t)q * S] = a;
            mine += (a < 0);
        }
        if (mine) atomicAdd(&s_unassigned, mine);
        __syncthreads();
        if (tid == 0 && p.stats_out) {
            if (s_unassigned) atomicAdd(reinterpret_cast<unsigned long long*>(p.stats_out + 4 * b + 3),
                                        (unsigned long long)s_unassigned);
            if (c == 0) {
                p.stats_out[4 * b + 0] = rounds;
                p.stats_out[4 * b + 1] = rowbids;
            }
        }
        if (c == 0) {
            R* pout = reinterpret_cast<R*>(p.prices_out) + b * p.M;
            for (int j = tid; j < M; j += blockDim.x) pout[j] = Ps[j];
        }
        __syncthreads();
    }
    if (tid == 0 && s_err) atomicCAS(p.status, ELA_OK, s_err);
}

}  // namespace

// ================================================================ host side
namespace {

unsigned long long g_wait_ns = 2000000000ull;
int g_skip_arrive = 0;

struct Plan {
    int path;            // ELA_PATH_CTA or ELA_PATH_GRID
    int S, ngroups, rpc; // grid path
    size_t smem;         // dynamic shared memory per CTA
    size_t group_bytes;  // grid path
    size_t ws_bytes;     // total workspace
};

int elem_size(int dtype) {
    switch (dtype) {
    case ELA_DTYPE_F32: return 4;
    case ELA_DTYPE_F16: return 2;
    case ELA_DTYPE_BF16: return 2;
    case ELA_DTYPE_F64: return 8;
    default: return 0;
    }
}

template <typename R>
int make_plan_t(int64_t B, int64_t N, int64_t M, int path, int sms, size_t smem_max, Plan& pl) {
    const int warps = ELA_CTA_THREADS / 32;
    const size_t cta_smem = cta_layout<R>(N, M, warps).total;
    const bool cta_fits = cta_smem <= smem_max;
    // grid plan
    const int T = sms;  // one CTA per SM
    int ngroups = (int)(B < T ? B : T);
    if (ngroups < 1) ngroups = 1;
    int S = T / ngroups;
    if (S > N) S = (int)(N > 0 ? N : 1);
    if (S < 1) S = 1;
    const int rpc = (int)((N + S - 1) / S);
    const size_t grid_smem_b = grid_smem<R>(M, rpc, ELA_GRID_THREADS / 32).total;
    const bool grid_fits = rpc <= ELA_ROWS_PER_CTA_MAX && grid_smem_b <= smem_max;

    int chosen = path;
    if (path == ELA_PATH_AUTO) {
        if (cta_fits && (N <= 512 || B >= sms)) chosen = ELA_PATH_CTA;
        else if (grid_fits) chosen = ELA_PATH_GRID;
        else if (cta_fits) chosen = ELA_PATH_CTA;
        else return ELA_ERR_UNSUPPORTED;
    }
    pl.path = chosen;
    if (chosen == ELA_PATH_CTA) {
        if (!cta_fits) return ELA_ERR_UNSUPPORTED;
        pl.S = 1; pl.ngroups = 0; pl.rpc = 0;
        pl.smem = cta_smem;
        pl.group_bytes = 0;
        pl.ws_bytes = ELA_WS_HEADER;
    } else if (chosen == ELA_PATH_GRID) {
        if (!grid_fits) return ELA_ERR_UNSUPPORTED;
        pl.S = S; pl.ngroups = ngroups; pl.rpc = rpc;
        pl.smem = grid_smem_b;
        pl.group_bytes = group_layout<R>(N, M).total;
        pl.ws_bytes = ELA_WS_HEADER + (size_t)ngroups * pl.group_bytes;
    } else {
        return ELA_ERR_ARGUMENT;
    }
    return ELA_OK;
}

int device_limits(int& sms, size_t& smem_max) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ELA_ERR_CUDA;
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return ELA_ERR_CUDA;
    sms = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return ELA_ERR_CUDA;
    smem_max = (size_t)v - 1024;  // room for the kernels' static shared variables
    return ELA_OK;
}

int make_plan(int dtype, int64_t B, int64_t N, int64_t M, int path, Plan& pl) {
    if (elem_size(dtype) == 0 || B < 0 || N < 0 || M < 0) return ELA_ERR_ARGUMENT;
    if (path < ELA_PATH_AUTO || path > ELA_PATH_GRID) return ELA_ERR_ARGUMENT;
    if (N > 0 && M < 2) return ELA_ERR_ARGUMENT;
    if (N >= (1ll << 30) || M >= (1ll << 30)) return ELA_ERR_UNSUPPORTED;
    int sms = 0;
    size_t smem_max = 0;
    const int rc = device_limits(sms, smem_max);
    if (rc != ELA_OK) return rc;
    return dtype == ELA_DTYPE_F64 ? make_plan_t<double>(B, N, M, path, sms, smem_max, pl)
                                  : make_plan_t<float>(B, N, M, path, sms, smem_max, pl);
}

template <typename In, typename R>
int launch(const Params& p, const Plan& pl, cudaStream_t stream) {
    if (pl.path == ELA_PATH_CTA) {
        auto kern = auction_cta_kernel<In, R>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess)
            return ELA_ERR_CUDA;
        const int64_t grid = p.B < (1ll << 20) ? p.B : (1ll << 20);
        kern<<<(unsigned int)grid, ELA_CTA_THREADS, pl.smem, stream>>>(p);
        return cudaGetLastError() == cudaSuccess ? ELA_OK : ELA_ERR_CUDA;
    }
    auto kern = auction_grid_kernel<In, R>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess)
        return ELA_ERR_CUDA;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, ELA_GRID_THREADS, pl.smem) != cudaSuccess)
        return ELA_ERR_CUDA;
    if (occ < 1) return ELA_ERR_UNSUPPORTED;
    // Every CTA of a group waits on the others, so all of them must be resident:
    // the cooperative launch refuses a grid that cannot be co-scheduled.
    Params pc = p;
    void* args[] = {&pc};
    const cudaError_t e = cudaLaunchCooperativeKernel((const void*)kern, dim3(pl.S * pl.ngroups),
                                                      dim3(ELA_GRID_THREADS), args, pl.smem, stream);
    return e == cudaSuccess ? ELA_OK : ELA_ERR_CUDA;
}

}  // namespace

extern "C" {

int ela_auction_version(void) { return 100; }

const char* ela_status_string(int status) {
    switch (status) {
    case ELA_OK: return "ok";
    case ELA_ERR_ARGUMENT: return "invalid argument";
    case ELA_ERR_CUDA: return "CUDA error";
    case ELA_ERR_TIMEOUT: return "device-side wait timed out";
    case ELA_ERR_UNSUPPORTED: return "unsupported size for this build";
    case ELA_ERR_INTERNAL: return "device-side consistency check failed";
    default: return "unknown status";
    }
}

size_t ela_auction_workspace_bytes(int dtype, int64_t B, int64_t N, int64_t M, int path) {
    Plan pl;
    if (make_plan(dtype, B, N, M, path, pl) != ELA_OK) return 0;
    return pl.ws_bytes;
}

void ela_auction_set_wait_limit_ns(uint64_t ns) { g_wait_ns = ns ? ns : 1; }

void ela_auction_debug_skip_arrive(int on) { g_skip_arrive = on ? 1 : 0; }

int ela_auction_solve(const void* cost, int dtype, int64_t B, int64_t N, int64_t M,
                      int64_t stride_b, int64_t stride_n, const double* eps_schedule,
                      int n_eps, int max_iter, int path, int64_t* assign_out,
                      void* prices_out, int64_t* stats_out, int32_t* status_out,
                      void* workspace, size_t workspace_bytes, void* stream) {
    const int es = elem_size(dtype);
    if (es == 0 || B < 0 || N < 0 || M < 0 || max_iter < 0) return ELA_ERR_ARGUMENT;
    if (n_eps < 1 || n_eps > ELA_MAX_PHASES || eps_schedule == nullptr) return ELA_ERR_ARGUMENT;
    for (int k = 0; k < n_eps; ++k)
        if (!(eps_schedule[k] > 0.0) || eps_schedule[k] == INFINITY) return ELA_ERR_ARGUMENT;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (B == 0 || N == 0) {
        if (B > 0 && M > 0 && prices_out &&
            cudaMemsetAsync(prices_out, 0, (size_t)(B * M) * (dtype == ELA_DTYPE_F64 ? 8 : 4), s) != cudaSuccess)
            return ELA_ERR_CUDA;
        if (stats_out && B > 0 && cudaMemsetAsync(stats_out, 0, (size_t)B * 32, s) != cudaSuccess)
            return ELA_ERR_CUDA;
        if (status_out && cudaMemsetAsync(status_out, 0, 4, s) != cudaSuccess) return ELA_ERR_CUDA;
        return ELA_OK;
    }
    if (!cost || !assign_out || !prices_out || !workspace) return ELA_ERR_ARGUMENT;
    if (stride_n < M || (B > 1 && stride_b < (N - 1) * stride_n + M)) return ELA_ERR_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return ELA_ERR_ARGUMENT;
    Plan pl;
    int rc = make_plan(dtype, B, N, M, path, pl);
    if (rc != ELA_OK) return rc;
    if (workspace_bytes < pl.ws_bytes) return ELA_ERR_ARGUMENT;

    Params p;
    memset(&p, 0, sizeof(p));
    p.cost = cost;
    p.B = B; p.N = N; p.M = M; p.stride_b = stride_b; p.stride_n = stride_n;
    for (int k = 0; k < n_eps; ++k) p.eps[k] = eps_schedule[k];
    p.n_eps = n_eps;
    p.max_iter = max_iter;
    p.vec_ok = ((reinterpret_cast<uintptr_t>(cost) & 15u) == 0) && ((stride_n * es) % 16 == 0) &&
               ((stride_b * es) % 16 == 0) && ((M * es) % 16 == 0);
    p.assign_out = assign_out;
    p.prices_out = prices_out;
    p.stats_out = stats_out;
    unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
    p.status = status_out ? status_out : reinterpret_cast<int32_t*>(ws + 4);
    p.ws = ws;
    p.group_bytes = pl.group_bytes;
    p.S = pl.S;
    p.ngroups = pl.ngroups;
    p.rows_per_cta = pl.rpc;
    p.wait_ns = g_wait_ns;
    p.skip_arrive = g_skip_arrive;

    if (cudaMemsetAsync(workspace, 0, pl.ws_bytes, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (status_out && cudaMemsetAsync(status_out, 0, 4, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (stats_out && cudaMemsetAsync(stats_out, 0, (size_t)B * 32, s) != cudaSuccess) return ELA_ERR_CUDA;

    switch (dtype) {
    case ELA_DTYPE_F32: return launch<float, float>(p, pl, s);
    case ELA_DTYPE_F16: return launch<__half, float>(p, pl, s);
    case ELA_DTYPE_BF16: return launch<__nv_bfloat16, float>(p, pl, s);
    default: return launch<double, double>(p, pl, s);
    }
}

}  // extern "C"
