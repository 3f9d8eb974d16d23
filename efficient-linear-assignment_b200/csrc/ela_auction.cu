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
// One kernel, two layouts of the work:
//   S == 1   each CTA solves whole problems; all state in shared memory.
//   S  > 1   S co-resident CTAs share one problem (cooperative launch); every
//            CTA keeps the full price vector and replays each round's election
//            from the round's complete bid list, which the CTAs exchange
//            through tagged words in global memory (the exchange is also the
//            round's only synchronisation between CTAs).
// The C ABI is declared in include/ela_auction.h.

#include <cuda_runtime.h>
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>
#include <unordered_map>
#include <type_traits>

#include "ela_auction.h"

#define ELA_MAX_PHASES 32
#define ELA_SMALL_M 128           // below this torch.topk uses introselect

#ifdef ELA_PROF
__device__ unsigned long long g_prof[16];
__device__ unsigned long long g_trace[8192][12];
#define PROF_MARK(var) long long var = clock64()
#define PROF_ADDALL(slot, v) do { if (threadIdx.x == 0 && MULTI) atomicAdd(&g_prof[slot], (unsigned long long)(v)); } while (0)
#define PROF_ADD(slot, a, b) do { if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(&g_prof[slot], (unsigned long long)((b) - (a))); } while (0)
#else
#define PROF_MARK(var)
#define PROF_ADD(slot, a, b)
#define PROF_ADDALL(slot, v)
#endif

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

// Election key of a row among the bids within 1e-5 of a column's new price;
// the largest key wins (atomicMax), 0 means no winner.  ELA_TIE_HIGHEST_ROW is
// the reference's rule (index_put_ with ascending rows keeps the last writer,
// torch_backend.py:126-136); ELA_TIE_LOWEST_ROW keeps the first.
__device__ __forceinline__ int win_key(int row, int N, int rule) { return rule == ELA_TIE_LOWEST_ROW ? N - row : row + 1; }

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

// 16-byte load through the read-only path (the cost matrix is never written
// during a solve).  Lines may stay in L1: a CTA re-reads the rows it owns,
// and in small rounds the same column slices, round after round.
__device__ __forceinline__ uint4 ld_stream16(const void* ptr) {
    uint4 r;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(ptr));
    return r;
}

// ------------------------------------------------------- cost sources
// Where the scans' cost values come from.  NoSum: the cost tensor.
// WithSum<In>: the target cost of the IMLE backward, cost + lam * grad,
// rounded as torch evaluates it in the input dtype (lam * grad rounded to the
// dtype, then the sum rounded), read from the two tensors (same strides;
// gdiff = byte distance from a cost element to the matching grad element)
// instead of a materialised sum.
struct NoSum {
    __device__ __forceinline__ uint4 load(const uint4* ptr) const { return ld_stream16(ptr); }
    template <typename In, typename R> __device__ __forceinline__ R one(const In* ptr) const {
        return Elem<In>::template one<R>(ptr);
    }
};

template <typename In> struct SumOps;
template <> struct SumOps<float> {
    static __device__ __forceinline__ unsigned int add(unsigned int c, unsigned int g, double lam) {
        return __float_as_uint(__fadd_rn(__uint_as_float(c), __fmul_rn((float)lam, __uint_as_float(g))));
    }
    static __device__ __forceinline__ float one(float c, float g, double lam) { return __fadd_rn(c, __fmul_rn((float)lam, g)); }
};
template <> struct SumOps<double> {
    static __device__ __forceinline__ double one(double c, double g, double lam) { return __dadd_rn(c, __dmul_rn(lam, g)); }
};
template <> struct SumOps<__half> {
    static __device__ __forceinline__ float one(float c, float g, double lam) {
        const float t = __half2float(__float2half_rn(__fmul_rn((float)lam, g)));
        return __half2float(__float2half_rn(__fadd_rn(c, t)));
    }
    static __device__ __forceinline__ unsigned short add(unsigned short c, unsigned short g, double lam) {
        __half_raw hc, hg, hr;
        hc.x = c; hg.x = g;
        hr = __half_raw(__float2half_rn(one(__half2float(__half(hc)), __half2float(__half(hg)), lam)));
        return hr.x;
    }
};
template <> struct SumOps<__nv_bfloat16> {
    static __device__ __forceinline__ float bf(unsigned short h) { return __uint_as_float(((unsigned int)h) << 16); }
    static __device__ __forceinline__ float one(float c, float g, double lam) {
        const float t = __bfloat162float(__float2bfloat16_rn(__fmul_rn((float)lam, g)));
        return __bfloat162float(__float2bfloat16_rn(__fadd_rn(c, t)));
    }
    static __device__ __forceinline__ unsigned short add(unsigned short c, unsigned short g, double lam) {
        return (unsigned short)(__float_as_uint(one(bf(c), bf(g), lam)) >> 16);  // one() is exact in bf16
    }
};

template <typename In> struct WithSum {
    long long gdiff;  // bytes from a cost element to the matching grad element
    double lam;
    __device__ __forceinline__ uint4 load(const uint4* ptr) const {
        const uint4 c = ld_stream16(ptr);
        const uint4 g = ld_stream16(reinterpret_cast<const char*>(ptr) + gdiff);
        if constexpr (std::is_same<In, float>::value) {
            return make_uint4(SumOps<float>::add(c.x, g.x, lam), SumOps<float>::add(c.y, g.y, lam),
                              SumOps<float>::add(c.z, g.z, lam), SumOps<float>::add(c.w, g.w, lam));
        } else if constexpr (std::is_same<In, double>::value) {
            const double c0 = __longlong_as_double((long long)(((unsigned long long)c.y << 32) | c.x));
            const double c1 = __longlong_as_double((long long)(((unsigned long long)c.w << 32) | c.z));
            const double g0 = __longlong_as_double((long long)(((unsigned long long)g.y << 32) | g.x));
            const double g1 = __longlong_as_double((long long)(((unsigned long long)g.w << 32) | g.z));
            const unsigned long long r0 = (unsigned long long)__double_as_longlong(SumOps<double>::one(c0, g0, lam));
            const unsigned long long r1 = (unsigned long long)__double_as_longlong(SumOps<double>::one(c1, g1, lam));
            return make_uint4((unsigned int)r0, (unsigned int)(r0 >> 32), (unsigned int)r1, (unsigned int)(r1 >> 32));
        } else {
            const unsigned int cw[4] = {c.x, c.y, c.z, c.w}, gw[4] = {g.x, g.y, g.z, g.w};
            unsigned int r[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const unsigned int lo = SumOps<In>::add((unsigned short)(cw[k] & 0xffffu), (unsigned short)(gw[k] & 0xffffu), lam);
                const unsigned int hi = SumOps<In>::add((unsigned short)(cw[k] >> 16), (unsigned short)(gw[k] >> 16), lam);
                r[k] = lo | (hi << 16);
            }
            return make_uint4(r[0], r[1], r[2], r[3]);
        }
    }
    template <typename In2, typename R> __device__ __forceinline__ R one(const In2* ptr) const {
        const R c = Elem<In2>::template one<R>(ptr);
        const R g = Elem<In2>::template one<R>(reinterpret_cast<const In2*>(reinterpret_cast<const char*>(ptr) + gdiff));
        return (R)SumOps<In2>::one(c, g, lam);
    }
};

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

template <typename R> __device__ __forceinline__ R rmax(R a, R b) { return a > b ? a : b; }
template <typename R> __device__ __forceinline__ R rmin(R a, R b) { return a < b ? a : b; }
template <> __device__ __forceinline__ float rmax<float>(float a, float b) { return fmaxf(a, b); }
template <> __device__ __forceinline__ float rmin<float>(float a, float b) { return fminf(a, b); }

template <typename R> __device__ __forceinline__ void top2_add(Top2<R>& t, R v, int col) {
    // branch-free (selects and min/max only), so the lanes of a warp never
    // diverge here; values are never NaN (finite costs and prices)
    const bool gt = (v > t.v1) || (t.p1 < 0);
    const bool eq = (v == t.v1);
    t.v2 = gt ? t.v1 : rmax(t.v2, v);
    t.p2 = gt ? -1 : ((eq && t.p2 < 0) ? col : t.p2);
    t.v1 = gt ? v : t.v1;
    t.p1 = gt ? col : t.p1;
}

// Merge two disjoint column sets; commutative, so a butterfly leaves every
// lane with the same result.  Selects only (no branches), so the lanes of a
// warp never diverge in the butterflies: the larger maximum keeps its state
// (its second value raised to the other maximum); equal maxima make a tie whose
// two columns are the two smallest of the candidates; an empty side (p1 < 0)
// yields the other side.
template <typename R> __device__ __forceinline__ Top2<R> top2_merge(Top2<R> a, Top2<R> b) {
    const bool gt = a.v1 > b.v1, lt = b.v1 > a.v1;
    const int big = 0x7fffffff;
    const int ap2 = a.p2 >= 0 ? a.p2 : big, bp2 = b.p2 >= 0 ? b.p2 : big;
    const bool af = a.p1 < b.p1;
    const int p1e = af ? a.p1 : b.p1;
    const int q1 = af ? ap2 : bp2, q2 = af ? b.p1 : a.p1;
    const int p2e = q1 < q2 ? q1 : q2;
    const R av2 = (a.v2 > b.v1) ? a.v2 : b.v1, bv2 = (b.v2 > a.v1) ? b.v2 : a.v1;
    Top2<R> r;
    r.v1 = lt ? b.v1 : a.v1;
    r.v2 = gt ? av2 : (lt ? bv2 : a.v1);
    r.p1 = gt ? a.p1 : (lt ? b.p1 : p1e);
    r.p2 = gt ? a.p2 : (lt ? b.p2 : p2e);
    r = (b.p1 < 0) ? a : r;
    r = (a.p1 < 0) ? b : r;
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

// fp32: the same reduction with warp-wide integer reductions (redux.sync) on
// order-preserving keys of the values.  -0 and +0 compare equal in the
// reference's comparisons, so both map to the key of +0.
__device__ __forceinline__ unsigned int fkey(float v) {
    unsigned int u = __float_as_uint(v + 0.0f);  // -0 + +0 = +0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(unsigned int k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
template <> __device__ __forceinline__ Top2<float> top2_warp<float>(Top2<float> t) {
    const int big = 0x7fffffff;
    const bool live = t.p1 >= 0;
    const unsigned int k1 = live ? fkey(t.v1) : 0u;
    const unsigned int K1 = __reduce_max_sync(0xffffffffu, k1);
    const bool top = live && k1 == K1;
    // independent of one another once K1 is known:
    const int P1 = (int)__reduce_min_sync(0xffffffffu, (unsigned int)(top ? t.p1 : big));
    const unsigned int k2 = !live ? 0u : (top ? (t.v2 == -INFINITY ? 0u : fkey(t.v2)) : k1);
    const unsigned int K2 = __reduce_max_sync(0xffffffffu, k2);
    const unsigned int topmask = __ballot_sync(0xffffffffu, top);
    const bool tie = (__popc(topmask) >= 2) || __any_sync(0xffffffffu, top && t.p2 >= 0);
    Top2<float> r;
    r.p1 = (K1 == 0u) ? -1 : P1;
    r.v1 = (K1 == 0u) ? -INFINITY : fkey_inv(K1);
    r.p2 = -1;
    r.v2 = (K2 == 0u) ? -INFINITY : fkey_inv(K2);
    if (tie) {  // rare: the maximum occurs twice; find its second column
        const int own2 = (t.p2 >= 0) ? t.p2 : big;
        const int cand = top ? ((t.p1 == P1) ? own2 : t.p1) : big;
        r.p2 = (int)__reduce_min_sync(0xffffffffu, (unsigned int)cand);
        r.v2 = r.v1;
    }
    return r;
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
    unsigned char* ws;       // workspace: header + exchange segments
    size_t seg_bytes;        // bytes of one CTA's exchange segment (S > 1)
    int S;                   // CTAs per problem
    int ngroups;             // problems in flight (S > 1)
    int rows_per_cta;        // ceil(N / S)
    unsigned long long wait_ns;
    int skip_publish;        // test hook: CTA 0 never publishes its first round
    int max_wpr;             // most warps that share one row's scan (power of two)
    int team;                // cluster path: clusters per problem
    int tie_rule;            // ELA_TIE_*: which row wins among bids within 1e-5 of the new price
    // virtual padding (ela_auction_solve_padded): the problem is N x M, the cost
    // tensor holds its first Nr rows and Mr columns; the other entries are
    // pad_c (real row x pad column, pad row x real column) or dd_c (pad row x
    // pad column), never stored.  vpad == 0: no padding (Nr == N, Mr == M).
    int vpad;
    int64_t Nr, Mr;
    double pad_c, dd_c;
    // fused IMLE target (ela_auction_solve_sum): the costs are cost + lam * grad,
    // grad at byte distance gdiff from cost with the same strides
    int gsum;
    long long gdiff;
    double lam;
    int cache_k;             // one-CTA path: row-cache entries per row (0: no cache)
    size_t team_bytes;       // cluster path: workspace bytes per team
};

// Row i of the current problem, or nullptr for a virtual padding row.
template <typename In>
__device__ __forceinline__ const In* row_ptr(const Params& p, const In* base, int64_t i) {
    return (p.vpad && i >= p.Nr) ? nullptr : base + i * p.stride_n;
}

// What the row scans need of the launch parameters, passed by value: an
// out-of-line scan given a reference to the kernel's parameters would make
// the kernel keep a local copy of all of them.
struct RowGeo {
    int M, vec_ok, vpad, Mr;
    double pad_c, dd_c;
};
__device__ __forceinline__ RowGeo row_geo(const Params& p) {
    return RowGeo{(int)p.M, p.vec_ok, p.vpad, (int)p.Mr, p.pad_c, p.dd_c};
}
// The cluster kernel's rows: no virtual padding (compile-time), two registers.
struct PlainGeo {
    int M, vec_ok;
    static constexpr int vpad = 0, Mr = 0;
    static constexpr double pad_c = 0.0, dd_c = 0.0;
};
__device__ __forceinline__ PlainGeo plain_geo(const Params& p) { return PlainGeo{(int)p.M, p.vec_ok}; }

// Cost of column `col` of a row (scalar load; the row pointer is nullptr for a
// padding row), with the padding blocks of ela_auction_solve_padded.
template <typename In, typename R, typename S = NoSum, typename G = RowGeo>
__device__ __forceinline__ R cost_at(const G& p, const In* row, int col, const S& src = S()) {
    if (!p.vpad) return src.template one<In, R>(row + col);
    if (row != nullptr) return col < p.Mr ? src.template one<In, R>(row + col) : (R)p.pad_c;
    return col < p.Mr ? (R)p.pad_c : (R)p.dd_c;
}

// ------------------------------------------------------------ row scanning
// W consecutive prices from shared memory (one or two vector loads).
template <typename R, int W> __device__ __forceinline__ void load_prices(const R* Ps, int c0, R* out) {
    if (sizeof(R) * W == 16) {
        const float4 q = *reinterpret_cast<const float4*>(Ps + c0);
        const R* r = reinterpret_cast<const R*>(&q);
#pragma unroll
        for (int e = 0; e < W; ++e) out[e] = r[e];
    } else if (sizeof(R) * W == 32) {
        const float4 q0 = *reinterpret_cast<const float4*>(Ps + c0);
        const float4 q1 = *(reinterpret_cast<const float4*>(Ps + c0) + 1);
        const R* r0 = reinterpret_cast<const R*>(&q0);
        const R* r1 = reinterpret_cast<const R*>(&q1);
#pragma unroll
        for (int e = 0; e < W / 2; ++e) { out[e] = r0[e]; out[W / 2 + e] = r1[e]; }
    } else {
#pragma unroll
        for (int e = 0; e < W; ++e) out[e] = Ps[c0 + e];
    }
}

#ifndef ELA_PF_BATCHES
#define ELA_PF_BATCHES 1  // L2 prefetch distance of the row scans, in batches
#endif

// L2 prefetch of this warp's chunks PF batches after the batch at `base`
// (lane's chunk; the warp's chunks of slot u are the 32 consecutive chunks
// from base - lane + u*stride, i.e. four 128-byte lines).  Lane l < 4*UNROLL
// takes line l % 4 of slot l / 4.  Costs no registers beyond the address.
template <int UNROLL, bool PF>
__device__ __forceinline__ void prefetch_batch(const uint4* rv, int base, int stride, int nchunks) {
    if (ELA_PF_BATCHES > 0 && PF) {
        const int lane = threadIdx.x & 31;
        if (lane < 4 * UNROLL) {
            const int ch = base - lane + ELA_PF_BATCHES * UNROLL * stride + (lane >> 2) * stride + (lane & 3) * 8;
            if (ch < nchunks) asm volatile("prefetch.global.L2 [%0];" ::"l"(rv + ch));
        }
    }
}

// One 16-byte chunk added to the lane's exact top-2.  A chunk whose maximum is
// not above the running second value cannot change it (a tied maximum is
// already recorded whenever v2 == v1), so only other chunks pay per element.
template <typename In, typename R>
__device__ __forceinline__ void exact_chunk(const uint4& raw, const R* __restrict__ Ps, int ch, Top2<R>& t) {
    constexpr int W = Elem<In>::W;
    R x[W], pr[W], v[W];
    Elem<In>::template unpack<R>(raw, x);
    load_prices<R, W>(Ps, ch * W, pr);
#pragma unroll
    for (int e = 0; e < W; ++e) v[e] = sub_rn(-x[e], pr[e]);
    R cm = v[0];
#pragma unroll
    for (int e = 1; e < W; ++e) cm = rmax(cm, v[e]);
    if (t.p1 < 0 || cm > t.v2) {
#pragma unroll
        for (int e = 0; e < W; ++e) top2_add(t, v[e], ch * W + e);
    }
}

#ifndef ELA_EXACT16
#define ELA_EXACT16 1  // 16-bit costs in the cluster kernel: exact scans only (1: large rounds, 2: all rounds)
#endif

// Lane-local exact top-2 over chunks base, base+stride, ... below nchunks
// (16-byte vectors of W elements).  Whole batches of UNROLL loads run without
// bounds predicates; the last, partial batch is predicated.
template <typename In, typename R, int UNROLL, bool PF, typename S = NoSum>
__device__ __forceinline__ void scan_chunks(const uint4* rv, const R* __restrict__ Ps, int base, int stride,
                                            int nchunks, Top2<R>& t, const S& src = S()) {
    for (; base + (UNROLL - 1) * stride < nchunks; base += stride * UNROLL) {
        uint4 raw[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) raw[u] = src.load(rv + base + u * stride);
        prefetch_batch<UNROLL, PF>(rv, base, stride, nchunks);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) exact_chunk<In, R>(raw[u], Ps, base + u * stride, t);
    }
    if (UNROLL > 1 && base < nchunks) {
        uint4 raw[UNROLL > 1 ? UNROLL - 1 : 1];
#pragma unroll
        for (int u = 0; u < UNROLL - 1; ++u)
            if (base + u * stride < nchunks) raw[u] = src.load(rv + base + u * stride);
#pragma unroll
        for (int u = 0; u < UNROLL - 1; ++u)
            if (base + u * stride < nchunks) exact_chunk<In, R>(raw[u], Ps, base + u * stride, t);
    }
}

// ---- fast scan: (v1, p1, v2) only.  A tied maximum shows as v1 == v2 after
// the warp reduction; only then is the row scanned again with exact tie
// tracking (scan_row).  Within a 16-byte chunk the top-2 is a pairwise tree of
// independent min/max operations; only the merge into the lane state is serial.
template <typename R, int W>
__device__ __forceinline__ void chunk_top2(const R* v, R& mx, R& sd, int& ix) {
    R m[W], n[W];
    int i[W];
#pragma unroll
    for (int e = 0; e < W; ++e) { m[e] = v[e]; n[e] = -INFINITY; i[e] = e; }
#pragma unroll
    for (int w = W; w > 1; w >>= 1) {
#pragma unroll
        for (int e = 0; e < w / 2; ++e) {
            const R a = m[2 * e], b = m[2 * e + 1];
            const bool right = b > a;  // ties keep the earlier column
            const R nn = rmax(rmin(a, b), rmax(n[2 * e], n[2 * e + 1]));
            i[e] = right ? i[2 * e + 1] : i[2 * e];
            m[e] = rmax(a, b);
            n[e] = nn;
        }
    }
    mx = m[0]; sd = n[0]; ix = i[0];
}

template <typename R>
__device__ __forceinline__ void lane_merge(Top2<R>& t, R mx, R sd, int col) {
    const bool gt = (mx > t.v1) || (t.p1 < 0);
    t.v2 = gt ? rmax(t.v1, sd) : rmax(t.v2, mx);
    t.p1 = gt ? col : t.p1;
    t.v1 = gt ? mx : t.v1;
}

#ifndef ELA_UNROLL_FAST
#define ELA_UNROLL_FAST 4  // loads in flight per lane in the fast scan (8 spills in the cluster kernel)
#endif

// One 16-byte chunk folded into the lane state, branch-free: with 32 lanes
// some lane almost always holds a chunk that beats its running second value,
// so a per-chunk filter branch costs the warp more than it saves.
template <typename In, typename R>
__device__ __forceinline__ void fast_chunk(const uint4& raw, const R* __restrict__ Ps, int ch, Top2<R>& t) {
    constexpr int W = Elem<In>::W;
    R x[W], pr[W], v[W];
    Elem<In>::template unpack<R>(raw, x);
    load_prices<R, W>(Ps, ch * W, pr);
#pragma unroll
    for (int e = 0; e < W; ++e) v[e] = sub_rn(-x[e], pr[e]);
    R mx, sd;
    int ix;
    chunk_top2<R, W>(v, mx, sd, ix);
    lane_merge(t, mx, sd, ch * W + ix);
}

// Chunks base, base+stride, ... below nchunks.  Whole batches of UNROLL loads
// run without bounds predicates; the last, partial batch is predicated.
template <typename In, typename R, int UNROLL, typename S = NoSum>
__device__ __forceinline__ void scan_chunks_fast(const uint4* rv, const R* __restrict__ Ps, int base, int stride,
                                                 int nchunks, Top2<R>& t, const S& src = S()) {
    for (; base + (UNROLL - 1) * stride < nchunks; base += stride * UNROLL) {
        uint4 raw[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) raw[u] = src.load(rv + base + u * stride);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) fast_chunk<In, R>(raw[u], Ps, base + u * stride, t);
    }
    if (UNROLL > 1 && base < nchunks) {
        uint4 raw[UNROLL > 1 ? UNROLL - 1 : 1];
#pragma unroll
        for (int u = 0; u < UNROLL - 1; ++u)
            if (base + u * stride < nchunks) raw[u] = src.load(rv + base + u * stride);
#pragma unroll
        for (int u = 0; u < UNROLL - 1; ++u)
            if (base + u * stride < nchunks) fast_chunk<In, R>(raw[u], Ps, base + u * stride, t);
    }
}

// Warp reduction of fast states; p2 stays -1 (v1 == v2 marks a tie).
template <typename R> __device__ __forceinline__ Top2<R> top2_warp_fast(Top2<R> t) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        Top2<R> o;
        o.v1 = __shfl_xor_sync(0xffffffffu, t.v1, off);
        o.v2 = __shfl_xor_sync(0xffffffffu, t.v2, off);
        o.p1 = __shfl_xor_sync(0xffffffffu, t.p1, off);
        if (o.p1 >= 0) {
            if (t.p1 < 0) { t = o; }
            else {
                const bool ob = (o.v1 > t.v1) || (o.v1 == t.v1 && o.p1 < t.p1);
                const R lo = ob ? t.v1 : o.v1;
                t.v2 = rmax(rmax(t.v2, o.v2), lo);
                if (ob) { t.v1 = o.v1; t.p1 = o.p1; }
            }
        }
    }
    t.p2 = -1;
    return t;
}
template <> __device__ __forceinline__ Top2<float> top2_warp_fast<float>(Top2<float> t) {
    const int big = 0x7fffffff;
    const bool live = t.p1 >= 0;
    const unsigned int k1 = live ? fkey(t.v1) : 0u;
    const unsigned int K1 = __reduce_max_sync(0xffffffffu, k1);
    const bool top = live && k1 == K1;
    const int P1 = (int)__reduce_min_sync(0xffffffffu, (unsigned int)(top ? t.p1 : big));
    // second value: a second lane at the maximum, the top lane's own second,
    // or the best other lane
    const unsigned int k2 = !live ? 0u : ((top && t.p1 == P1) ? (t.v2 == -INFINITY ? 0u : fkey(t.v2)) : k1);
    const unsigned int K2 = __reduce_max_sync(0xffffffffu, k2);
    Top2<float> r;
    r.p1 = (K1 == 0u) ? -1 : P1;
    r.v1 = (K1 == 0u) ? -INFINITY : fkey_inv(K1);
    r.v2 = (K2 == 0u) ? -INFINITY : fkey_inv(K2);
    r.p2 = -1;
    return r;
}

template <typename In, typename R, typename S = NoSum, typename G = RowGeo>
__device__ __forceinline__ Top2<R> scan_row_fast(const G p, const In* row, const R* __restrict__ Ps,
                                                 int lane, int sub, int wpr, const S& src = S()) {
    const int M = (int)p.M;
    Top2<R> t;
    top2_init(t);
    if (p.vec_ok) {
        constexpr int W = Elem<In>::W;
        const int nchunks = M / W;
        const int stride = 32 * wpr;
        const int per_lane = (nchunks + stride - 1) / stride;
        const uint4* rv = reinterpret_cast<const uint4*>(row);
        const int base = sub * 32 + lane;
        if (per_lane <= 1) scan_chunks_fast<In, R, 1>(rv, Ps, base, stride, nchunks, t, src);
        else if (per_lane <= 2) scan_chunks_fast<In, R, 2>(rv, Ps, base, stride, nchunks, t, src);
        else if (per_lane <= 4) scan_chunks_fast<In, R, 4>(rv, Ps, base, stride, nchunks, t, src);
        else scan_chunks_fast<In, R, ELA_UNROLL_FAST>(rv, Ps, base, stride, nchunks, t, src);
    } else {
        for (int col = sub * 32 + lane; col < M; col += 32 * wpr)
            lane_merge(t, sub_rn(-cost_at<In, R>(p, row, col, src), Ps[col]), (R)-INFINITY, col);
    }
    return top2_warp_fast(t);
}

// Fast scans of two rows by one warp at once (16-byte aligned rows): the
// loads of both rows are in flight together, so a warp that owns several rows
// in a round waits one memory latency per pair instead of per row.  Each row's
// state is the one scan_row_fast computes.  `two` is warp-uniform.
template <typename In, typename R, typename S = NoSum, typename G = RowGeo>
__device__ __forceinline__ void scan_rows2_fast(const G p, const In* ra, const In* rb, bool two,
                                                const R* __restrict__ Ps, int lane, Top2<R>& ta, Top2<R>& tb,
                                                const S& src = S()) {
    constexpr int W = Elem<In>::W, U = 4;
    const int nchunks = (int)p.M / W;
    const uint4* va = reinterpret_cast<const uint4*>(ra);
    const uint4* vb = reinterpret_cast<const uint4*>(rb);
    top2_init(ta);
    top2_init(tb);
    int base = lane;
    for (; base + (U - 1) * 32 < nchunks; base += 32 * U) {
        uint4 a[U], b[U];
#pragma unroll
        for (int u = 0; u < U; ++u) a[u] = src.load(va + base + u * 32);
        if (two) {
#pragma unroll
            for (int u = 0; u < U; ++u) b[u] = src.load(vb + base + u * 32);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) fast_chunk<In, R>(a[u], Ps, base + u * 32, ta);
        if (two) {
#pragma unroll
            for (int u = 0; u < U; ++u) fast_chunk<In, R>(b[u], Ps, base + u * 32, tb);
        }
    }
    for (; base < nchunks; base += 32) {
        const uint4 a = src.load(va + base);
        uint4 b = a;
        if (two) b = src.load(vb + base);
        fast_chunk<In, R>(a, Ps, base, ta);
        if (two) fast_chunk<In, R>(b, Ps, base, tb);
    }
    ta = top2_warp_fast(ta);
    if (two) tb = top2_warp_fast(tb);
}

// Top-2 over the columns of one row that this warp covers: the row's 16-byte
// chunks are dealt to `wpr` warps in turn (warp `sub` takes chunks
// sub*32+lane, sub*32+lane+32*wpr, ...).  The batch size follows the number
// of chunks per lane, so no predicated-off batch slots are issued.  The
// result is reduced over the warp.
template <typename In, typename R, typename S = NoSum, typename G = RowGeo>
__device__ __noinline__ Top2<R> scan_row(const G p, const In* row, const R* __restrict__ Ps,
                                         int lane, int sub, int wpr, const S src = S()) {
    const int M = (int)p.M;
    Top2<R> t;
    top2_init(t);
    if (p.vec_ok) {
        constexpr int W = Elem<In>::W;
        const int nchunks = M / W;
        const int stride = 32 * wpr;
        const int per_lane = (nchunks + stride - 1) / stride;
        const uint4* rv = reinterpret_cast<const uint4*>(row);
        const int base = sub * 32 + lane;
        if (per_lane <= 1) scan_chunks<In, R, 1, false>(rv, Ps, base, stride, nchunks, t, src);
        else if (per_lane <= 2) scan_chunks<In, R, 2, false>(rv, Ps, base, stride, nchunks, t, src);
        else scan_chunks<In, R, 4, true>(rv, Ps, base, stride, nchunks, t, src);
    } else {
        for (int col = sub * 32 + lane; col < M; col += 32 * wpr)
            top2_add(t, sub_rn(-cost_at<In, R>(p, row, col, src), Ps[col]), col);
    }
    return top2_warp(t);
}

// scan_row for the cluster kernel (no padding, no fused sum): it takes the
// launch parameters by reference, which keeps that kernel's calls as lean as
// they were before the padding and sum variants existed (measured: 4 % of a
// cfg2 solve against the by-value geometry).
template <typename In, typename R>
__device__ __noinline__ Top2<R> scan_row_plain(const Params& p, const In* row, const R* __restrict__ Ps,
                                         int lane, int sub, int wpr) {
    const int M = (int)p.M;
    Top2<R> t;
    top2_init(t);
    if (p.vec_ok) {
        constexpr int W = Elem<In>::W;
        const int nchunks = M / W;
        const int stride = 32 * wpr;
        const int per_lane = (nchunks + stride - 1) / stride;
        const uint4* rv = reinterpret_cast<const uint4*>(row);
        const int base = sub * 32 + lane;
        if (per_lane <= 1) scan_chunks<In, R, 1, false>(rv, Ps, base, stride, nchunks, t);
        else if (per_lane <= 2) scan_chunks<In, R, 2, false>(rv, Ps, base, stride, nchunks, t);
        else scan_chunks<In, R, 4, true>(rv, Ps, base, stride, nchunks, t);
    } else {
        for (int col = sub * 32 + lane; col < M; col += 32 * wpr)
            top2_add(t, sub_rn(-Elem<In>::template one<R>(row + col), Ps[col]), col);
    }
    return top2_warp(t);
}

// Column choice and bid from the row's complete top-2 (whole warp, uniform).
template <typename In, typename R, typename S = NoSum, typename G = RowGeo>
__device__ __forceinline__ void finish_bid(const G p, const In* row, const R* __restrict__ Ps,
                                           const Top2<R>& t, R eps, int lane, R* scr_v, int* scr_i,
                                           int& j1_out, R& bid_out, const S& src = S()) {
    const int M = (int)p.M;
    int j1;
    if (t.v1 == t.v2 && M < ELA_SMALL_M) {
        for (int col = lane; col < M; col += 32) {
            scr_v[col] = sub_rn(-cost_at<In, R>(p, row, col, src), Ps[col]);
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

// ------------------------------------------------------------- row cache
// Prices never fall during a solve (a new price is the column's maximum bid,
// never below the old price, and each epsilon phase starts from the previous
// phase's prices), and fl((-c) - P) is non-increasing in P, so every value
// v[j] of a row only falls.  After a full scan of row i the cache keeps the
// entries S = {(j, c[i][j]) : v[j] > tau}; tau bounds every column outside S
// then, and so at every later time.  A later bid of the row recomputes the
// values of S with the current prices: if their second value is still above
// tau, the row's exact top-2 lies in S, including every occurrence of a tied
// maximum (all of them are above tau), so the bid equals a full scan's.
// Otherwise the row is scanned again and S rebuilt.  One warp per row; at
// most 64 entries, lane l holding entries l and l + 32.

// Top-2 of row i from its cache (exact, ties included); true if it is the
// row's top-2 (second value above the cache's bound).
template <typename R, bool TWO>
__device__ __forceinline__ bool cache_top2_t(const R* __restrict__ Ps, const unsigned short* ccol, const R* ccost,
                                             int n, R tau, int lane, Top2<R>& t) {
    top2_init(t);
    if (lane < n) {
        const int j = ccol[lane];
        t.v1 = sub_rn(-ccost[lane], Ps[j]);
        t.p1 = j;
    }
    if (TWO && lane + 32 < n) {  // entries are in no column order: merge (ties keep the two smallest columns)
        Top2<R> u;
        top2_init(u);
        const int j = ccol[lane + 32];
        u.v1 = sub_rn(-ccost[lane + 32], Ps[j]);
        u.p1 = j;
        t = top2_merge(t, u);
    }
    t = top2_warp(t);
    return t.v2 > tau;
}
template <typename R>
__device__ __forceinline__ bool cache_top2(const R* __restrict__ Ps, const unsigned short* ccol, const R* ccost,
                                           int n, R tau, int lane, Top2<R>& t) {
    return n > 32 ? cache_top2_t<R, true>(Ps, ccol, ccost, n, tau, lane, t)
                  : cache_top2_t<R, false>(Ps, ccol, ccost, n, tau, lane, t);
}

// Full scan of a row of M = NCH*32*W columns held in registers (lane l has the
// 16-byte chunks l, l+32, ...), exact top-2 with ties, then a new cache: the
// threshold search looks for the lowest tau with at most kc values above it
// (interpolating the count between a bound that holds too many and one that
// holds few enough; every lane's maximum exceeds the lowest lane maximum, so
// that bound starts the search), then the values above tau are compacted into
// the cache with ballots.
template <typename In, int NCH, typename S = NoSum>
__device__ __noinline__ Top2<float> scan_build(const In* row, const float* __restrict__ Ps, int lane, int kc,
                                               unsigned short* ccol, float* ccost, float* ctau, unsigned char* ccnt,
                                               const S src = S()) {
    constexpr int W = Elem<In>::W, NV = NCH * W;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    uint4 raw[NCH];
#pragma unroll
    for (int u = 0; u < NCH; ++u) raw[u] = src.load(rv + lane + 32 * u);
    float v[NV];
    Top2<float> t;
    top2_init(t);
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
        float x[W], pr[W];
        Elem<In>::template unpack<float>(raw[u], x);
        load_prices<float, W>(Ps, (lane + 32 * u) * W, pr);
#pragma unroll
        for (int e = 0; e < W; ++e) {
            v[u * W + e] = sub_rn(-x[e], pr[e]);
            top2_add(t, v[u * W + e], (lane + 32 * u) * W + e);
        }
    }
    const unsigned int lane_max_key = fkey(t.v1);
    const Top2<float> r = top2_warp(t);
    auto count_above = [&](float th) {
        int c = 0;
#pragma unroll
        for (int k = 0; k < NV; ++k) c += (v[k] > th) ? 1 : 0;
        return (int)__reduce_add_sync(0xffffffffu, (unsigned int)c);
    };
    float hi = r.v1, lo = fkey_inv(__reduce_min_sync(0xffffffffu, lane_max_key));
    int hic = 0, loc = count_above(lo);
    if (loc <= kc) {
        hi = lo;
        hic = loc;
    } else {
        const float target = 0.95f * (float)kc;
        for (int it = 0; it < 6; ++it) {
            float th = hi - (hi - lo) * ((target - (float)hic) / (float)(loc - hic));
            if (!(th > lo && th < hi)) th = 0.5f * (lo + hi);
            const int m = count_above(th);
            if (m <= kc) {
                hi = th;
                hic = m;
                if (m >= kc - kc / 8) break;
            } else {
                lo = th;
                loc = m;
            }
        }
    }
    int base = 0;
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
        float x[W];
        Elem<In>::template unpack<float>(raw[u], x);
#pragma unroll
        for (int e = 0; e < W; ++e) {
            const bool keep = v[u * W + e] > hi;
            const unsigned int m = __ballot_sync(0xffffffffu, keep);
            if (keep) {
                const int pos = base + __popc(m & ((1u << lane) - 1u));
                ccol[pos] = (unsigned short)((lane + 32 * u) * W + e);
                ccost[pos] = x[e];
            }
            base += __popc(m);
        }
    }
    if (lane == 0) { *ctau = hi; *ccnt = (unsigned char)hic; }
    return r;
}

// One cached row's bid (one warp): from the cache when it still holds the
// row's top-2, else from a full scan that rebuilds the cache.  Rows of
// nch * 32 16-byte chunks, nch <= 32 / W (at most 32 values per lane).
// Returns the column bid on; *bid_out gets the bid.
template <typename In, typename S = NoSum>
__device__ __noinline__ int cached_row_bid(int nch, const In* row, const float* __restrict__ Ps, float eps, int lane,
                                           int kc, unsigned short* ccol, float* ccost, float* ctau,
                                           unsigned char* ccnt, float* bid_out, const S src = S()) {
    constexpr int W = Elem<In>::W;
    Top2<float> tt;
    const int n = *ccnt;
    bool hit = false;
    if (n >= 2) hit = cache_top2<float>(Ps, ccol, ccost, n, *ctau, lane, tt);
    if (!hit) {
        switch (nch) {
        case 1: tt = scan_build<In, 1, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src); break;
        case 2: tt = scan_build<In, 2, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src); break;
        case 3: tt = scan_build<In, 3, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src); break;
        default:
            if constexpr (W == 4) {
                switch (nch) {
                case 4: tt = scan_build<In, 4, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src); break;
                case 5: tt = scan_build<In, 5, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src); break;
                case 6: tt = scan_build<In, 6, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src); break;
                case 7: tt = scan_build<In, 7, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src); break;
                default: tt = scan_build<In, 8, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src); break;
                }
            } else {
                tt = scan_build<In, 4, S>(row, Ps, lane, kc, ccol, ccost, ctau, ccnt, src);
            }
        }
    }
    const int j1 = (tt.p2 >= 0 && !(tt.p1 == 0 && tt.p2 == 1)) ? tt.p2 : tt.p1;
    *bid_out = add_rn(Ps[j1], add_rn(sub_rn(tt.v1, tt.v2), eps));
    return j1;
}

// One row's bid by one warp from a full scan (exact top-2 on a tied
// maximum); returns the column, *bid_out the bid.  Out of line: it serves the
// one-bidder chains of the one-CTA kernel, whose registers stay free.
template <typename In, typename R, typename S = NoSum, typename G = RowGeo>
__device__ __noinline__ int plain_row_bid(const G p, const In* row, const R* __restrict__ Ps, R eps, int lane,
                                          R* scr_v, int* scr_i, R* bid_out, const S src = S()) {
    Top2<R> tt = scan_row_fast<In, R, S>(p, row, Ps, lane, 0, 1, src);
    if (p.M >= ELA_SMALL_M && tt.v1 == tt.v2) tt = scan_row<In, R, S>(p, row, Ps, lane, 0, 1, src);
    int j1;
    finish_bid<In, R, S>(p, row, Ps, tt, eps, lane, scr_v, scr_i, j1, *bid_out, src);
    return j1;
}

// ------------------------------------------------------ bid exchange (S > 1)
// Each CTA of a group publishes its round-t bids in its own segment of the
// round's buffer (two buffers, by round parity):
//   word 0                 header  (t+1) << 32 | count
//   words 1+EW*k ...       entry k: A = (t+1)&0xffff << 48 | row << 24 | col,
//                          then the bid bits in 32-bit halves, each under a
//                          32-bit copy of t+1.
// Every word carries the round tag, so a reader needs no fence: it re-reads
// any word whose tag is not yet the current round's.  Reading all S segments
// of round t is also the round's barrier.  A CTA cannot publish round t+2
// (reusing the buffer) before every CTA has published round t+1, which each
// does only after it has read all of round t.
template <typename R> struct Ex;
template <> struct Ex<float> { static constexpr int EW = 2, INL = 3; };
template <> struct Ex<double> { static constexpr int EW = 3, INL = 2; };

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* ptr) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(ptr) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* ptr, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(ptr), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_u32(unsigned int* ptr, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* ptr) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

template <typename R>
__device__ __forceinline__ void put_entry(unsigned long long* seg, int k, unsigned int t1, int row, int col, R bid) {
    unsigned long long* w = seg + 1 + Ex<R>::EW * k;
    const unsigned long long tag = (unsigned long long)t1 << 32;
    st_relaxed_u64(w, ((unsigned long long)(t1 & 0xffffu) << 48) | ((unsigned long long)row << 24) | (unsigned long long)col);
    const unsigned long long bits = (unsigned long long)Bits<R>::to(bid);
    st_relaxed_u64(w + 1, tag | (bits & 0xffffffffull));
    if (Ex<R>::EW == 3) st_relaxed_u64(w + 2, tag | (bits >> 32));
}

template <typename R>
__device__ __forceinline__ bool entry_tags_ok(const unsigned long long* w, unsigned int t1) {
    if ((w[0] >> 48) != (t1 & 0xffffu) || (unsigned int)(w[1] >> 32) != t1) return false;
    return Ex<R>::EW == 2 || (unsigned int)(w[2] >> 32) == t1;
}
template <typename R>
__device__ __forceinline__ void decode_entry(const unsigned long long* w, int& row, int& col, R& bid) {
    row = (int)((w[0] >> 24) & 0xffffffull);
    col = (int)(w[0] & 0xffffffull);
    const unsigned long long hi = (Ex<R>::EW == 3) ? w[2] : 0ull;
    const unsigned long long bits = (w[1] & 0xffffffffull) | ((hi & 0xffffffffull) << 32);
    bid = Bits<R>::from((typename Bits<R>::U)bits);
}

// One attempt to read entry k; false if some word is not yet from round t1.
template <typename R>
__device__ __forceinline__ bool get_entry(const unsigned long long* seg, int k, unsigned int t1, int& row, int& col,
                                          R& bid) {
    const unsigned long long* w = seg + 1 + Ex<R>::EW * k;
    const unsigned long long a = ld_relaxed_u64(w);
    const unsigned long long lo = ld_relaxed_u64(w + 1);
    const unsigned long long hi = (Ex<R>::EW == 3) ? ld_relaxed_u64(w + 2) : 0ull;
    if ((a >> 48) != (t1 & 0xffffu) || (unsigned int)(lo >> 32) != t1) return false;
    if (Ex<R>::EW == 3 && (unsigned int)(hi >> 32) != t1) return false;
    row = (int)((a >> 24) & 0xffffffull);
    col = (int)(a & 0xffffffull);
    const unsigned long long bits = (lo & 0xffffffffull) | ((hi & 0xffffffffull) << 32);
    bid = Bits<R>::from((typename Bits<R>::U)bits);
    return true;
}


// Reads every entry past the inline ones of the S segments of round t1,
// spread over the whole CTA (one L2 latency, not one per segment).  cnt/off:
// per-segment counts and list offsets; exoff: S+1 ints of shared scratch.
// Returns false if an entry never showed up (status and abort flag are set).
template <typename R, typename IX = int>
__device__ bool read_extra_entries(const unsigned char* segbase, size_t seg_bytes, int S, const int* cnt,
                                   const int* off, int* exoff, unsigned int t1, R* lbid, IX* lrow, IX* lcol,
                                   int* abort_flag, int32_t* status) {
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < 32) {  // exclusive prefix of the extra counts, one warp
        const int per = (S + 31) / 32, a = lane * per, b = min(S, a + per);
        int sum = 0;
        for (int sg = a; sg < b; ++sg) sum += max(0, cnt[sg] - Ex<R>::INL);
        int x = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        int run = x - sum;
        for (int sg = a; sg < b; ++sg) { exoff[sg] = run; run += max(0, cnt[sg] - Ex<R>::INL); }
        if (lane == 31) exoff[S] = x;
    }
    __syncthreads();
    const int total = exoff[S];
    bool ok = true;
    constexpr int BATCH = 4;  // entries per thread whose loads are in flight together
    for (int b0 = tid; b0 < total && ok; b0 += BATCH * blockDim.x) {
        int seg_of[BATCH], k_of[BATCH];
        unsigned long long w[BATCH][Ex<R>::EW];
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
            const int idx = b0 + u * blockDim.x;
            seg_of[u] = -1;
            if (idx < total) {
                int lo = 0, hi = S - 1;  // last segment whose extra entries start at or before idx
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (exoff[mid] <= idx) lo = mid; else hi = mid - 1;
                }
                seg_of[u] = lo;
                k_of[u] = Ex<R>::INL + (idx - exoff[lo]);
                const unsigned long long* e = reinterpret_cast<const unsigned long long*>(segbase + (size_t)lo * seg_bytes) +
                                              1 + Ex<R>::EW * k_of[u];
#pragma unroll
                for (int q = 0; q < Ex<R>::EW; ++q) w[u][q] = ld_relaxed_u64(e + q);
            }
        }
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
            if (seg_of[u] < 0) continue;
            const unsigned long long* seg = reinterpret_cast<const unsigned long long*>(segbase + (size_t)seg_of[u] * seg_bytes);
            int rr = 0, cc = 0;
            R bb = (R)0;
            if (entry_tags_ok<R>(w[u], t1)) {
                decode_entry<R>(w[u], rr, cc, bb);
            } else {  // not visible yet: re-read this entry until its words carry the tag
                unsigned int tries = 0;
                while (!get_entry<R>(seg, k_of[u], t1, rr, cc, bb)) {
                    if (++tries > (1u << 22)) {
                        atomicCAS(status, ELA_OK, ELA_ERR_TIMEOUT);
                        atomicExch(abort_flag, 1);
                        ok = false;
                        break;
                    }
                }
            }
            const int o = off[seg_of[u]] + k_of[u];
            lbid[o] = bb; lrow[o] = (IX)rr; lcol[o] = (IX)cc;
        }
    }
    return __syncthreads_and(ok) != 0;
}

// ================================================================== kernel
// Shared-memory layout (byte offsets), identical on host and device.
struct KLayout {
    size_t P, maxb, win, owner, lbid, lrow, lcol, rowcol, rowbid, active, wtop, scr_v, scr_i;
    size_t ccol, ccost, ctau, ccnt;  // row cache (kc > 0)
    size_t total;
};
__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

template <typename R>
__host__ __device__ inline KLayout k_layout(int64_t N, int64_t M, int rpc, int warps, int kc = 0) {
    KLayout L;
    size_t o = 0;
    L.P = o;      o = align_up(o + sizeof(R) * (size_t)M, 16);   // prices
    L.maxb = o;   o = align_up(o + sizeof(R) * (size_t)M, 16);   // round's column max bid (bits)
    L.win = o;    o = align_up(o + 4 * (size_t)M, 16);           // round's elected row + 1
    L.owner = o;  o = align_up(o + 4 * (size_t)M, 16);           // one-CTA path: row owning each column
    L.lbid = o;   o = align_up(o + sizeof(R) * (size_t)N, 16);   // round's bids: value
    L.lrow = o;   o = align_up(o + 4 * (size_t)N, 16);           //               row
    L.lcol = o;   o = align_up(o + 4 * (size_t)N, 16);           //               column
    L.rowcol = o; o = align_up(o + 4 * (size_t)rpc, 16);         // own rows: assigned column or -1
    L.rowbid = o; o = align_up(o + 4 * (size_t)rpc, 16);         // own rows: column bid on, or -1
    L.active = o; o = align_up(o + 4 * (size_t)rpc, 16);         // own rows bidding this round
    L.wtop = o;   o = align_up(o + (2 * sizeof(R) + 8) * (size_t)warps, 16);  // per-warp top-2
    const size_t scr = (M < ELA_SMALL_M) ? (size_t)warps * ELA_SMALL_M : 0;
    L.scr_v = o;  o = align_up(o + sizeof(R) * scr, 16);
    L.scr_i = o;  o = align_up(o + 4 * scr, 16);
    L.ccost = o;  o = align_up(o + sizeof(R) * (size_t)rpc * kc, 16);  // row cache: cost of each entry
    L.ccol = o;   o = align_up(o + 2 * (size_t)rpc * kc, 16);          //             column of each entry
    L.ctau = o;   o = align_up(o + sizeof(R) * (size_t)(kc ? rpc : 0), 16);  // bound on every other column
    L.ccnt = o;   o = align_up(o + (size_t)(kc ? rpc : 0), 16);        //             entries (0: none)
    L.total = o;
    return L;
}

// Launch shapes: one CTA per problem runs 256 threads at up to 2 CTAs per SM
// (a batch of small problems stays in one wave); the multi-CTA path runs 512
// threads, one CTA per SM.
#define ELA_THREADS_ONE 256
#ifndef ELA_MINB_ONE
#define ELA_MINB_ONE 2
#endif
#define ELA_THREADS_MULTI 512
#ifndef ELA_THREADS_CLUSTER
#define ELA_THREADS_CLUSTER 512  // threads per CTA of the cluster kernel
#endif
#define ELA_MINB_MULTI 1
#define ELA_MAX_S 256
#define ELA_WS_HEADER 256

// Round: active rows bid -> bids gathered -> column max (new price) -> highest
// row within 1e-5 of it wins -> owners of bid-on columns are evicted.
//   MULTI == false: every CTA solves whole problems (blockIdx.x, +gridDim.x, ...);
//                   a round's bids go straight into the CTA's shared list.
//   MULTI == true:  S CTAs share a problem; CTA c owns the block of rows
//                   [c*rpc, (c+1)*rpc), rpc = ceil(N/S) (few TLB pages per CTA)
template <typename In, typename R, bool MULTI, int THREADS, int MINB, bool CACHE = false, typename S = NoSum>
__global__ void __launch_bounds__(THREADS, MINB)
auction_kernel(const Params p) {
    static_assert(!CACHE || (!MULTI && std::is_same<R, float>::value), "row cache: one-CTA path, fp32 prices");
    typedef Bits<R> BT;
    typedef typename BT::U U;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int s_nact, s_total, s_extra, s_fail;
    __shared__ int s_ties, s_exact;  // rows whose maximum tied; scan exactly first when many do
    __shared__ int s_cnt[MULTI ? ELA_MAX_S : 1], s_off[MULTI ? ELA_MAX_S : 1];
    __shared__ int s_exoff[MULTI ? ELA_MAX_S + 1 : 1];
    __shared__ int s_unassigned;
    __shared__ int s_chain;  // one-bidder rounds run by warp 0 alone

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    S src;  // cost source: the cost tensor, or cost + lam * grad (IMLE backward target)
    if constexpr (!std::is_same<S, NoSum>::value) {
        src.gdiff = p.gdiff;
        src.lam = p.lam;
    }
    const int SG = MULTI ? p.S : 1;
    const int g = blockIdx.x / SG, c = blockIdx.x % SG;
    const int N = (int)p.N, M = (int)p.M;
    const int row0 = c * p.rows_per_cta;                           // first owned row
    const int my_rows = (row0 < N) ? min(p.rows_per_cta, N - row0) : 0;
    const int kc = CACHE ? p.cache_k : 0;
    const KLayout L = k_layout<R>(N, M, p.rows_per_cta, nw, kc);
    R* P = reinterpret_cast<R*>(smem + L.P);
    U* maxb = reinterpret_cast<U*>(smem + L.maxb);
    int* win = reinterpret_cast<int*>(smem + L.win);
    int* owner = reinterpret_cast<int*>(smem + L.owner);  // maintained on the one-CTA path only
    R* lbid = reinterpret_cast<R*>(smem + L.lbid);
    int* lrow = reinterpret_cast<int*>(smem + L.lrow);
    int* lcol = reinterpret_cast<int*>(smem + L.lcol);
    int* rowcol = reinterpret_cast<int*>(smem + L.rowcol);
    int* rowbid = reinterpret_cast<int*>(smem + L.rowbid);
    int* active = reinterpret_cast<int*>(smem + L.active);
    Top2<R>* wtop = reinterpret_cast<Top2<R>*>(smem + L.wtop);
    R* scr_v = reinterpret_cast<R*>(smem + L.scr_v) + warp * ELA_SMALL_M;
    int* scr_i = reinterpret_cast<int*>(smem + L.scr_i) + warp * ELA_SMALL_M;
    const R tol = (R)1e-5;

    int* abort_flag = reinterpret_cast<int*>(p.ws);
    unsigned char* gbase = p.ws + ELA_WS_HEADER + (size_t)g * 2 * SG * p.seg_bytes;

    if (tid == 0) { s_ties = 0; s_exact = 0; }
    const int nprob_step = MULTI ? p.ngroups : gridDim.x;
    unsigned int t = 0;  // round counter, identical in all CTAs of a group
    bool first_publish = true;

    for (int64_t b = MULTI ? g : blockIdx.x; b < p.B; b += nprob_step) {
        const In* base = reinterpret_cast<const In*>(p.cost) + b * p.stride_b;
        for (int j = tid; j < M; j += blockDim.x) { P[j] = (R)0; maxb[j] = 0; win[j] = 0; owner[j] = -1; }
        for (int q = tid; q < my_rows; q += blockDim.x) { rowcol[q] = -1; rowbid[q] = -1; }
        if (kc)
            for (int q = tid; q < my_rows; q += blockDim.x) smem[L.ccnt + q] = 0;  // row caches empty
        long long rounds = 0, rowbids = 0;
        int ph = 0, it = 0;
        R eps = (R)p.eps[0];  // this epsilon (read once per epsilon)
        bool rebuild = true;  // the active list is rebuilt from rowcol at problem and epsilon starts
        __syncthreads();
        while (ph < p.n_eps) {
            if (it == p.max_iter) {  // round budget of this epsilon used up
                if (++ph < p.n_eps) {  // the next epsilon starts from unassigned rows
                    eps = (R)p.eps[ph];
                    for (int q = tid; q < my_rows; q += blockDim.x) rowcol[q] = -1;
                    for (int j = tid; j < M; j += blockDim.x) owner[j] = -1;
                }
                it = 0;
                rebuild = true;
                __syncthreads();
                continue;
            }
            const unsigned int t1 = t + 1;
            PROF_MARK(pt0);
            // ---- own rows that bid this round (otherwise listed by the last election)
            if (rebuild) {
                if (tid == 0) s_nact = 0;
                __syncthreads();
                for (int q = tid; q < my_rows; q += blockDim.x)
                    if (rowcol[q] < 0) active[atomicAdd(&s_nact, 1)] = q;
                rebuild = false;
            }
            if (tid == 0) { s_total = 0; s_extra = 0; s_fail = 0; }
            __syncthreads();
            const int K = s_nact;
            if constexpr (!MULTI) {
                if (K == 1) {
                    // ---- a chain of rounds with one bidder each, run by warp 0
                    //      alone (no CTA barrier, no election arrays): the only
                    //      bid sets the column's price (a bid never falls below
                    //      the old price) and wins it, and the evicted owner, if
                    //      any, is the next round's only bidder.  Identical to
                    //      running those rounds one by one.
                    if (warp == 0) {
                        int q = active[0], n = 0;
                        for (;;) {
                            const In* row = row_ptr(p, base, q);
                            int j1;
                            R bid;
#ifdef ELA_PROF
                            const long long c0 = clock64();
                            const int hit0 = CACHE ? 1 : 0;
#endif
                            if constexpr (CACHE) {
                                const KLayout LC = k_layout<R>(N, M, N, nw, kc);
                                const unsigned short* cc = reinterpret_cast<unsigned short*>(smem + LC.ccol) + (size_t)q * kc;
                                const float* cx = reinterpret_cast<float*>(smem + LC.ccost) + (size_t)q * kc;
                                // the cache hit, inline: each lane one entry, exact warp top-2
                                const int cn = smem[LC.ccnt + q];
                                Top2<float> tt;
                                const bool chit =
                                    cn >= 2 && cache_top2<float>(P, cc, cx, cn, reinterpret_cast<const float*>(smem + LC.ctau)[q], lane, tt);
                                if (chit) {
                                    j1 = (tt.p2 >= 0 && !(tt.p1 == 0 && tt.p2 == 1)) ? tt.p2 : tt.p1;
                                    bid = add_rn(P[j1], add_rn(sub_rn(tt.v1, tt.v2), eps));
#ifdef ELA_PROF
                                    if (lane == 0 && blockIdx.x == 0) {
                                        atomicAdd(&g_trace[8190][7], 1ull);
                                        atomicAdd(&g_trace[8190][8], (unsigned long long)(clock64() + (bid == 12345.f) - c0));
                                    }
#endif
                                } else {  // a miss: full scan and a new cache, out of line
                                    float fb;
                                    j1 = cached_row_bid<In, S>(M / (32 * Elem<In>::W), row, P, eps, lane, kc,
                                                            reinterpret_cast<unsigned short*>(smem + LC.ccol) + (size_t)q * kc,
                                                            reinterpret_cast<float*>(smem + LC.ccost) + (size_t)q * kc,
                                                            reinterpret_cast<float*>(smem + LC.ctau) + q, smem + LC.ccnt + q,
                                                            &fb, src);
                                    bid = fb;
                                }
                            } else {
                                j1 = plain_row_bid<In, R, S>(row_geo(p), row, P, eps, lane, scr_v, scr_i, &bid, src);
                            }
#ifdef ELA_PROF
                            const long long c1 = clock64() + (bid == (R)12345 ? 1 : 0);
#endif
                            const int prev = owner[j1];
                            __syncwarp();  // every lane has read P and owner before they change
                            if (lane == 0) {
                                P[j1] = bid;
                                owner[j1] = q;
                                rowcol[q] = j1;
                                if (prev >= 0) rowcol[prev] = -1;
                            }
                            __syncwarp();
#ifdef ELA_PROF
                            if (lane == 0 && blockIdx.x == 0) {
                                atomicAdd(&g_trace[8190][4], 1ull);
                                atomicAdd(&g_trace[8190][5], (unsigned long long)(c1 - c0));
                                atomicAdd(&g_trace[8190][6], (unsigned long long)(clock64() - c1));
                                (void)hit0;
                            }
#endif
                            ++n;
                            if (prev < 0 || it + n == p.max_iter) {
                                if (lane == 0) {
                                    s_nact = prev >= 0 ? 1 : 0;
                                    if (prev >= 0) active[0] = prev;
                                    s_chain = n;
                                }
                                break;
                            }
                            q = prev;
                        }
                    }
                    __syncthreads();
                    const int n = s_chain;
                    rounds += n;
                    rowbids += n;
                    it += n;
                    continue;
                }
            }
            PROF_MARK(pt1);
            unsigned long long* myseg =
                reinterpret_cast<unsigned long long*>(gbase + (size_t)((t & 1) * SG + c) * p.seg_bytes);
            // ---- bids against the round-start prices.  With few rows, a row is
            //      dealt to several warps so that its scan is one memory latency.
            if (K > 0) {
                // warps per row: the largest power of two with wpr * K <= nw
                // (nw is a power of two), as a shift
                int lw = 0;
                if (M >= 1024 && K < nw) {
                    const int lnw = 31 - __clz(nw);
                    const int lk = (K > 1) ? 32 - __clz(K - 1) : 0;  // ceil(log2 K)
                    lw = lnw - lk;
                    const int lmax = 31 - __clz(p.max_wpr);
                    if (lw > lmax) lw = lmax;
                }
                const int wpr = 1 << lw;
                const int groups = nw >> lw;
                // exact tie tracking is needed only when the maximum is tied
                // and M >= 128 (below that the tie is settled by introselect)
                const bool exact_ok = M >= ELA_SMALL_M;
                // a row's bid from its complete top-2: tie re-scan, column, entry
                auto emit = [&](int k, int q, const In* row, Top2<R> tt) {
                    if (exact_ok && tt.v1 == tt.v2) tt = scan_row<In, R, S>(row_geo(p), row, P, lane, 0, 1, src);
                    if (lane == 0 && tt.v1 == tt.v2) atomicAdd(&s_ties, 1);
                    int j1;
                    R bid;
                    finish_bid<In, R, S>(row_geo(p), row, P, tt, eps, lane, scr_v, scr_i, j1, bid, src);
                    if (lane == 0) {
                        rowbid[q] = j1;
                        if (!MULTI) { lbid[k] = bid; lrow[k] = row0 + q; lcol[k] = j1; }
                        else put_entry<R>(myseg, k, t1, row0 + q, j1, bid);
                    }
                };
                if constexpr (CACHE) {
                        // cached rows: a bid from the row's cache, else a full scan
                        // that rebuilds it (one warp per row)
                        const KLayout LC = k_layout<R>(N, M, N, nw, kc);
                        const int nch = M / (32 * Elem<In>::W);  // 16-byte chunks per lane of a cached row
                        for (int k = warp; k < K; k += nw) {
                            const int q = active[k];
                            float bid;
                            const int j1 = cached_row_bid<In, S>(
                                nch, base + (int64_t)q * p.stride_n, P, eps, lane, kc,
                                reinterpret_cast<unsigned short*>(smem + LC.ccol) + (size_t)q * kc,
                                reinterpret_cast<float*>(smem + LC.ccost) + (size_t)q * kc,
                                reinterpret_cast<float*>(smem + LC.ctau) + q, smem + LC.ccnt + q, &bid, src);
                            if (lane == 0) { rowbid[q] = j1; lbid[k] = bid; lrow[k] = q; lcol[k] = j1; }
                        }
                } else {
                if (lw == 0 && K > nw && !s_exact && p.vec_ok) {
                    // several rows per warp: two at a time (no CTA barrier in here)
                    for (int kb = 0; kb < K; kb += 2 * nw) {
                        const int ka = kb + warp, kb2 = ka + nw;
                        if (ka >= K) continue;
                        const bool two = kb2 < K;
                        const int qa = active[ka], qb = two ? active[kb2] : qa;
                        const In* ra = base + (int64_t)(row0 + qa) * p.stride_n;
                        const In* rb = base + (int64_t)(row0 + qb) * p.stride_n;
                        Top2<R> ta, tb;
                        scan_rows2_fast<In, R, S>(row_geo(p), ra, rb, two, P, lane, ta, tb, src);
                        emit(ka, qa, ra, ta);
                        if (two) emit(kb2, qb, rb, tb);
                    }
                } else
                for (int kb = 0; kb < K; kb += groups) {
                    const int k = kb + (warp >> lw), sub = warp & (wpr - 1);
                    const bool has = k < K;
                    const int q = has ? active[k] : 0;
                    const int i = row0 + q;
                    const In* row = row_ptr(p, base, i);
                    Top2<R> tt;
                    top2_init(tt);
                    const bool exact_first = (wpr == 1) && s_exact;  // tie-heavy rows: one exact pass
                    if (has) tt = exact_first ? scan_row<In, R, S>(row_geo(p), row, P, lane, 0, 1, src)
                                              : scan_row_fast<In, R, S>(row_geo(p), row, P, lane, sub, wpr, src);
#ifdef ELA_PROF
                    if (has && lane == 0 && t < 8192) atomicMax(&g_trace[t][8], (unsigned long long)(clock64() - pt1));
#endif
                    if (wpr > 1) {
                        if (has && lane == 0) wtop[warp] = tt;
                        __syncthreads();
                        const int gb = warp - sub;  // first warp of this row's group
                        if (has) {  // every warp of the group merges the group's partial results
                            Top2<R> o;
                            top2_init(o);
                            if (lane < wpr) o = wtop[gb + lane];
                            tt = top2_warp_fast(o);
                        }
                        const bool rowtie = exact_ok && has && tt.v1 == tt.v2;
                        if (__syncthreads_or(rowtie)) {  // also orders the wtop reads before rewrites
                            Top2<R> ex;
                            top2_init(ex);
                            if (rowtie) ex = scan_row<In, R, S>(row_geo(p), row, P, lane, sub, wpr, src);
                            if (rowtie && lane == 0) wtop[warp] = ex;
                            __syncthreads();
                            if (rowtie && sub == 0) {
                                Top2<R> o;
                                top2_init(o);
                                if (lane < wpr) o = wtop[gb + lane];
                                tt = top2_warp(o);
                            }
                        }
                    } else if (exact_ok && has && tt.v1 == tt.v2 && !exact_first) {
                        tt = scan_row<In, R, S>(row_geo(p), row, P, lane, 0, 1, src);
                    }
                    if (has && sub == 0 && lane == 0 && tt.v1 == tt.v2) atomicAdd(&s_ties, 1);
#ifdef ELA_PROF
                    if (has && sub == 0 && lane == 0 && t < 8192) atomicMax(&g_trace[t][9], (unsigned long long)(clock64() - pt1));
#endif
                    if (has && sub == 0) {
                        int j1;
                        R bid;
                        finish_bid<In, R, S>(row_geo(p), row, P, tt, eps, lane, scr_v, scr_i, j1, bid, src);
                        if (lane == 0) {
                            rowbid[q] = j1;
                            if (!MULTI) { lbid[k] = bid; lrow[k] = i; lcol[k] = j1; }
                            else put_entry<R>(myseg, k, t1, i, j1, bid);
#ifdef ELA_PROF
                            if (t < 8192) atomicMax(&g_trace[t][10], (unsigned long long)(clock64() - pt1));
#endif
                        }
                    }
                    if (wpr > 1 && kb + groups < K) __syncthreads();  // wtop is reused
                }
                }  // !CACHE
            }
            __syncthreads();
            if (tid == 0) { s_exact = (K > 0) ? (s_ties * 4 > K) : s_exact; s_ties = 0; }
            PROF_MARK(pt2);
            // ---- gather the round's bids of the whole problem
            int ntot;
            if (!MULTI) {
                ntot = K;
            } else {
                if (tid == 0 && !(p.skip_publish && first_publish && c == 0))
                    st_relaxed_u64(myseg, ((unsigned long long)t1 << 32) | (unsigned int)K);
                first_publish = false;
                if (tid < SG) {
                    const unsigned long long* seg =
                        reinterpret_cast<const unsigned long long*>(gbase + (size_t)((t & 1) * SG + tid) * p.seg_bytes);
                    const unsigned long long t0 = globaltimer_ns();
                    unsigned int spins = 0;
                    int cntv = -1;
                    constexpr int NW = 1 + Ex<R>::INL * Ex<R>::EW;
                    unsigned long long w[NW];
                    for (;;) {  // bounded wait: header and inline entries, loaded together
#pragma unroll
                        for (int k = 0; k < NW; ++k) w[k] = ld_relaxed_u64(seg + k);
                        if ((unsigned int)(w[0] >> 32) == t1) {
                            const int cn = (int)(unsigned int)(w[0] & 0xffffffffull);
                            bool ok = true;
#pragma unroll
                            for (int k = 0; k < Ex<R>::INL; ++k)
                                if (k < cn) ok = ok && entry_tags_ok<R>(w + 1 + Ex<R>::EW * k, t1);
                            if (ok) { cntv = cn; break; }
                        }
                        if ((++spins & 15u) == 0) {
                            if (*(volatile int*)abort_flag) break;
                            if (globaltimer_ns() - t0 > p.wait_ns) {
                                atomicExch(abort_flag, 1);
                                atomicCAS(p.status, ELA_OK, ELA_ERR_TIMEOUT);
                                break;
                            }
                        }
                    }
                    if (cntv < 0) {
                        s_fail = 1;
                    } else {
                        const int off = atomicAdd(&s_total, cntv);
                        s_cnt[tid] = cntv;
                        s_off[tid] = off;
                        if (cntv > Ex<R>::INL) s_extra = 1;
#pragma unroll
                        for (int k = 0; k < Ex<R>::INL; ++k)
                            if (k < cntv) {
                                int rr, cc;
                                R bb;
                                decode_entry<R>(w + 1 + Ex<R>::EW * k, rr, cc, bb);
                                lbid[off + k] = bb; lrow[off + k] = rr; lcol[off + k] = cc;
                            }
                    }
                }
                __syncthreads();
                PROF_MARK(pt2b);
                PROF_ADDALL(8, pt2b - pt2);
                if (s_fail) return;
                if (s_extra) {  // rounds with many bids: read the remaining entries together
                    if (!read_extra_entries<R>(gbase + (size_t)((t & 1) * SG) * p.seg_bytes, p.seg_bytes, SG, s_cnt,
                                               s_off, s_exoff, t1, lbid, lrow, lcol, abort_flag, p.status))
                        return;
                }
                ntot = s_total;
            }
            ++t;
            PROF_MARK(pt3);
            if (ntot == 0) {  // nobody bid: this epsilon's solve has converged
                rebuild = true;
                if (++ph < p.n_eps) {  // the next epsilon starts from unassigned rows
                    eps = (R)p.eps[ph];
                    for (int q = tid; q < my_rows; q += blockDim.x) rowcol[q] = -1;
                    for (int j = tid; j < M; j += blockDim.x) owner[j] = -1;
                }
                it = 0;
                __syncthreads();
                continue;
            }
            rounds++;
            rowbids += ntot;
            // ---- election, identical in every CTA of the group.  One CTA per
            //      problem with up to 32 bids: entry e is thread e of warp 0, warp
            //      barriers order the steps, and the next bidders (losers, and
            //      owners of the columns won) come from the entries instead of a
            //      pass over every row.
            if (!MULTI && ntot <= 32) {
                if (warp == 0) {
                    const bool valid = lane < ntot;
                    const int j = valid ? lcol[lane] : 0;
                    const int i = valid ? lrow[lane] : 0;  // row0 == 0 on this path
                    if (valid) atomicMax(&maxb[j], BT::to(lbid[lane]));
                    __syncwarp();
                    if (valid && absval(sub_rn(lbid[lane], BT::from(maxb[j]))) < tol) atomicMax(&win[j], win_key(i, N, p.tie_rule));
                    __syncwarp();
                    int nxt = -1;  // this entry's bidder in the next round
                    if (valid) {
                        nxt = i;  // lost: bids again
                        rowbid[i] = -1;
                        if (win[j] == win_key(i, N, p.tie_rule)) {
                            const int prev = owner[j];
                            if (prev >= 0) rowcol[prev] = -1;
                            owner[j] = i;
                            rowcol[i] = j;
                            nxt = prev;  // -1: took a free column
                        }
                        P[j] = BT::from(maxb[j]);
                    }
                    __syncwarp();  // every maxb[] / win[] read before they are cleared
                    if (valid) { maxb[j] = 0; win[j] = 0; }
                    const unsigned int m = __ballot_sync(0xffffffffu, nxt >= 0);
                    if (nxt >= 0) active[__popc(m & ((1u << lane) - 1))] = nxt;
                    if (lane == 0) s_nact = __popc(m);
                }
                __syncthreads();
            } else {
                // ---- election, identical in every CTA of the group
                for (int e = tid; e < ntot; e += blockDim.x) atomicMax(&maxb[lcol[e]], BT::to(lbid[e]));
                if (tid == 0) s_nact = 0;
                __syncthreads();
                for (int e = tid; e < ntot; e += blockDim.x) {
                    const int j = lcol[e];
                    if (absval(sub_rn(lbid[e], BT::from(maxb[j]))) < tol) atomicMax(&win[j], win_key(lrow[e], N, p.tie_rule));
                }
                __syncthreads();
                for (int q = tid; q < my_rows; q += blockDim.x) {
                    const int jb = rowbid[q];
                    int col = rowcol[q];
                    if (jb >= 0) {
                        col = (win[jb] == win_key(row0 + q, N, p.tie_rule)) ? jb : -1;
                        if (!MULTI && col >= 0) owner[col] = q;
                        rowbid[q] = -1;
                    } else if (col >= 0 && maxb[col] != 0) {
                        col = -1;  // someone took the column
                    }
                    rowcol[q] = col;
                    if (col < 0) active[atomicAdd(&s_nact, 1)] = q;  // bids next round
                }
                for (int e = tid; e < ntot; e += blockDim.x) P[lcol[e]] = BT::from(maxb[lcol[e]]);
                __syncthreads();
                // cleared before the next round's election; the bid phase's
                // barriers lie in between
                for (int e = tid; e < ntot; e += blockDim.x) { maxb[lcol[e]] = 0; win[lcol[e]] = 0; }
            }
            ++it;
            PROF_MARK(pt4);
            PROF_ADD(0, pt0, pt1); PROF_ADD(1, pt1, pt2); PROF_ADD(2, pt2, pt3); PROF_ADD(3, pt3, pt4);
            PROF_ADD(4, 0, 1); PROF_ADD(5, 0, (K > 0));
            if (K > 0) { PROF_ADDALL(6, pt2 - pt1); PROF_ADDALL(7, 1); PROF_ADDALL(10, K); }
            PROF_ADDALL(9, 1);
            PROF_ADDALL(11, pt3 - pt2);
#ifdef ELA_PROF
            if (t - 1 < 8192) {
                if (threadIdx.x == 0 && K > 0) atomicMax(&g_trace[t - 1][5], (unsigned long long)(pt2 - pt1));
                if (threadIdx.x == 0 && K > 0) atomicMax(&g_trace[t - 1][6], (unsigned long long)K);
                if (blockIdx.x == 0 && threadIdx.x == 0) {
                    g_trace[t - 1][0] = ntot; g_trace[t - 1][1] = pt1 - pt0; g_trace[t - 1][2] = pt2 - pt1;
                    g_trace[t - 1][3] = pt3 - pt2;
                    g_trace[t - 1][4] = pt4 - pt3;
                }
            }
#endif
        }
        // ---- outputs of problem b
        if (tid == 0) s_unassigned = 0;
        __syncthreads();
        int mine = 0;
        for (int q = tid; q < my_rows; q += blockDim.x) {
            const int a = rowcol[q];
            p.assign_out[b * p.N + row0 + q] = a;
            mine += (a < 0);
        }
        if (mine) atomicAdd(&s_unassigned, mine);
        if (c == 0) {
            R* pout = reinterpret_cast<R*>(p.prices_out) + b * p.M;
            for (int j = tid; j < M; j += blockDim.x) pout[j] = P[j];
        }
        __syncthreads();
        if (tid == 0 && p.stats_out) {
            if (s_unassigned)
                atomicAdd(reinterpret_cast<unsigned long long*>(p.stats_out + 4 * b + 3),
                          (unsigned long long)s_unassigned);
            if (c == 0) {
                p.stats_out[4 * b + 0] = rounds;
                p.stats_out[4 * b + 1] = rowbids;
            }
        }
        __syncthreads();
    }
}


// ============================================================ cluster kernel
// One thread-block cluster (CS CTAs, CS = 16 where the device allows it, else
// 8) per problem.  Every CTA holds the whole problem state in shared memory
// (prices, column owners, row assignments) and replays every round's election
// identically; the CTAs of the cluster exchange data through distributed
// shared memory (stores into the other CTAs' shared memory) and the cluster
// barrier.  Two kinds of rounds:
//   large rounds (K > ELA_SMALL_ROUND rows bid): each CTA scans its own block
//     of rows in full and stores its bids into every CTA's bid list;
//   small rounds: every CTA scans its 1/CS slice of the columns of all K
//     active rows and stores a partial top-2 per row into every CTA; each CTA
//     merges the CS partials of a row (the merge is exact, ties included), so
//     a row costs one memory latency instead of a full-row scan.
// The number of active rows never grows within an epsilon, so a solve runs
// large rounds, then small rounds, per epsilon.
// Per round: [scan] wait(consumed) [store to all CTAs] arrive+wait(ready)
// [merge, election] arrive(consumed).  The second barrier phase lets a CTA
// store the next round's data only after every CTA has read this round's.

#define ELA_SMALL_ROUND 64

struct CLayout {
    size_t P, win, owner, rowcol, act, lbid, lrow, lcol, part, cnt, evict, total;
};
// IX: index type of rows and columns in shared memory (16-bit when N and M
// are below 32768, which halves the footprint of the replicated state).
template <typename R, typename IX>
__host__ __device__ inline CLayout c_layout(int64_t N, int64_t M, int CS) {
    CLayout L;
    const int rpc = (int)((N + CS - 1) / CS);
    const size_t nlist = (size_t)rpc * CS;  // bid list: slot rank*rpc + k (DSMEM) or 0..K-1
    size_t o = 0;
    L.P = o;      o = align_up(o + sizeof(R) * (size_t)M, 16);   // prices (the round's max bid lands here)
    L.win = o;    o = align_up(o + 4 * (size_t)M, 16);           // elected row + 1 per column
    L.owner = o;  o = align_up(o + sizeof(IX) * (size_t)M, 16);  // row owning each column, -1
    L.rowcol = o; o = align_up(o + sizeof(IX) * (size_t)N, 16);  // column of each row, -1
    L.act = o;    o = align_up(o + sizeof(IX) * (size_t)N, 16);  // rows bidding this round, ascending
    L.lbid = o;   o = align_up(o + sizeof(R) * nlist, 16);
    L.lrow = o;   o = align_up(o + sizeof(IX) * nlist, 16);
    L.lcol = o;   o = align_up(o + sizeof(IX) * nlist, 16);
    L.part = o;   o = align_up(o + 2 * sizeof(Top2<R>) * (size_t)CS * ELA_SMALL_ROUND, 16);  // by round parity
    L.cnt = o;    o = align_up(o + 4 * (size_t)CS, 16);
    L.evict = o;  o = align_up(o + 4 * (size_t)ELA_SMALL_ROUND, 16);
    L.total = o;
    return L;
}

__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}


// ---- asynchronous stores into another CTA's shared memory, completed on
// that CTA's mbarrier (transaction bytes), and the local mbarrier wait.
__device__ __forceinline__ unsigned int smem_addr(const void* ptr) {
    return (unsigned int)__cvta_generic_to_shared(ptr);
}
__device__ __forceinline__ unsigned int cluster_map(unsigned int addr, int rank) {
    unsigned int r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_async_16(unsigned int raddr, uint4 v, unsigned int rmbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
                 ::"r"(raddr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rmbar) : "memory");
}
__device__ __forceinline__ void mbar_init(unsigned long long* mb, unsigned int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(mb)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* mb, unsigned int bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(mb)), "r"(bytes) : "memory");
}
// Bounded wait for phase `parity` of a local mbarrier; false on timeout or
// when *abort (the cluster's failure mark) is set.
__device__ __forceinline__ bool mbar_wait(unsigned long long* mb, unsigned int parity, unsigned long long limit_ns,
                                          const volatile int* abort) {
    const unsigned int a = smem_addr(mb);
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned int spins = 1;; ++spins) {
        unsigned int done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
        if ((spins & 15u) == 0) {  // slow path: a peer's failure mark, the time limit
            if (*abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) return false;
        }
    }
}

// One pass over the rows (ballots kept per lane) for 16-bit costs: cfg5-like
// solves whose late rounds have a few hundred bidders among 8192 rows spend
// half the cycles of the two-pass walk there (-3 % of the solve).  The fp32
// instance keeps the two-pass walk: with the one-pass code the 4096^2 fp32
// epsilon-schedule solve measured 3 % slower (code generation of its
// small-round loop, not the compaction itself, which runs ~50 times a solve).
#ifndef ELA_ONEPASS_COMPACT
#define ELA_ONEPASS_COMPACT(In) (sizeof(In) == 2)
#endif

#ifndef ELA_SPLIT_LARGE
#define ELA_SPLIT_LARGE 1  // 16-bit costs, large rounds with at most nw/2 rows per CTA: several warps per row
#endif

// Large rounds with few rows per CTA: warp w's share of row act[(w / wpr) * ST]
// (chunks strided over the row's wpr warps), top-2 into part[w]: exact
// (ties included) from one exact pass, or from the fast pass with an exact
// re-scan of a share whose maximum is tied.  Used for 16-bit costs only: in
// the fp32 cluster kernel the extra code spilled registers and cost the
// 4096^2 solve 17 %.
template <typename In, typename R, typename IX>
__device__ __forceinline__ void large_share(const PlainGeo g, int64_t stride_n, const In* base, const IX* act, int ST,
                                         int wpr, bool exact, const R* __restrict__ P, Top2<R>* part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kr = warp / wpr, sub = warp - kr * wpr;
    const In* row = base + (int64_t)act[kr * ST] * stride_n;
    Top2<R> tt;
    if (exact) {
        tt = scan_row<In, R, NoSum, PlainGeo>(g, row, P, lane, sub, wpr);
    } else {
        tt = scan_row_fast<In, R>(g, row, P, lane, sub, wpr);
        if (tt.p1 >= 0 && tt.v1 == tt.v2) tt = scan_row<In, R, NoSum, PlainGeo>(g, row, P, lane, sub, wpr);
    }
    if (lane == 0) part[warp] = tt;
}

// Block-wide ordered compaction of the rows with rowcol < 0 into act[];
// returns the count (all threads).  Deterministic: ascending row order.
template <typename IX, bool ONEPASS>
__device__ int compact_unassigned(const IX* rowcol, int N, IX* act, int* s_scan) {
    // Each warp owns a contiguous block of rows (a multiple of 32) and walks it
    // 32 rows at a time: consecutive lanes read consecutive entries (no bank
    // conflicts) and a ballot marks the unassigned rows.  Up to 32 ballots per
    // warp, lane k keeps the k-th, so the rows are read once; a warp scan of
    // the lanes' counts and the warps' totals place each lane's rows.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int per = (((N + nw - 1) / nw) + 31) & ~31;
    const int r0 = warp * per, r1 = min(N, r0 + per);
    if (ONEPASS && per <= 32 * 32) {
        unsigned int mine = 0u;
        int k = 0;
#pragma unroll 4
        for (int b = r0; b < r1; b += 32, ++k) {
            const int i = b + lane;
            const unsigned int m = __ballot_sync(0xffffffffu, i < r1 && rowcol[i] < 0);
            mine = (lane == k) ? m : mine;
        }
        const int c = __popc(mine);
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) s_scan[warp] = incl;
        __syncthreads();
        const unsigned int w = (lane < nw) ? (unsigned int)s_scan[lane] : 0u;
        int pos = (int)__reduce_add_sync(0xffffffffu, lane < warp ? w : 0u) + incl - c;
        const int total = (int)__reduce_add_sync(0xffffffffu, w);
        const int rb = r0 + 32 * lane;
        while (mine) {
            act[pos++] = (IX)(rb + __ffs(mine) - 1);
            mine &= mine - 1u;
        }
        __syncthreads();
        return total;
    }
    int cnt = 0;
    for (int b = r0; b < r1; b += 32) {
        const int i = b + lane;
        cnt += __popc(__ballot_sync(0xffffffffu, i < r1 && rowcol[i] < 0));
    }
    if (lane == 0) s_scan[warp] = cnt;
    __syncthreads();
    const unsigned int w = (lane < nw) ? (unsigned int)s_scan[lane] : 0u;
    int pos = (int)__reduce_add_sync(0xffffffffu, lane < warp ? w : 0u);  // rows of the warps before
    const int total = (int)__reduce_add_sync(0xffffffffu, w);
    const unsigned int below = (1u << lane) - 1u;
    for (int b = r0; b < r1; b += 32) {
        const int i = b + lane;
        const bool u = i < r1 && rowcol[i] < 0;
        const unsigned int m = __ballot_sync(0xffffffffu, u);
        if (u) act[pos + __popc(m & below)] = (IX)i;
        pos += __popc(m);
    }
    __syncthreads();
    return total;
}

// The cluster's failure exit (see the kernel): marks the abort flag, marks
// every peer's s_abort unless this CTA learned of the failure from its own,
// then arrives at and waits on the cluster barrier.  Kept out of line so that
// the round loop's code does not change for a path it never takes.
__device__ __noinline__ void cluster_leave(int* abort_flag, bool pending, int* s_abort, int CS) {
    const int tid = threadIdx.x;
    if (tid == 0) atomicExch(abort_flag, 1);
    if (pending) cluster_wait_acquire();
    if (tid < CS && !*(volatile int*)s_abort) {
        const unsigned int ra = cluster_map(smem_addr(s_abort), tid);
        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(ra), "r"(1) : "memory");
    }
    cluster_arrive_release();
    cluster_wait_acquire();
}

// Team layout: ngroups teams of p.team clusters; a team solves one problem at
// a time.  Large rounds use every CTA of the team (rows split over the team;
// bids exchanged through distributed shared memory when the team is one
// cluster, through tagged words in global memory otherwise).  Small rounds
// run in the team's first (leader) cluster only; the other clusters wait for
// the end of the epsilon and then reload the prices the leader publishes.
// Per-team workspace: [2 x ST exchange segments][prices M][flag word].
template <typename In, typename R, typename IX>
__global__ void __launch_bounds__(ELA_THREADS_CLUSTER, 1)
auction_cluster_kernel(const Params p) {
    namespace cg = cooperative_groups;
    typedef Bits<R> BT;
    typedef typename BT::U U;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int s_scan[32];
    __shared__ int s_cnt, s_total, s_extra, s_fail;
    __shared__ int s_ties, s_exact;  // rows whose maximum tied; scan exactly first when many do
    __shared__ int s_off[ELA_MAX_S + 1];
    __shared__ int s_segcnt[ELA_MAX_S];
    __shared__ int s_exoff[ELA_MAX_S + 1];
    __shared__ __align__(8) unsigned long long s_mbar[2];  // small-round partials, by round parity
    __shared__ int s_abort;  // some CTA of this cluster failed (set locally or by a peer through DSMEM)
    // fp32 partials are 16 bytes: one asynchronous store per destination CTA
    constexpr bool ASYNC = (sizeof(Top2<R>) == 16);

    cg::cluster_group cluster = cg::this_cluster();
    const int CS = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int cid = blockIdx.x / CS;
    const int TC = p.team;                    // clusters per team
    const int team = cid / TC, tc = cid % TC;
    const bool leader = (tc == 0);
    const int ST = TC * CS;                   // CTAs per team
    const int gi = tc * CS + rank;            // this CTA within the team
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int N = (int)p.N, M = (int)p.M;
    constexpr int W = Elem<In>::W;
    const int nchunks = M / W;
    const int rpc = (N + CS - 1) / CS;        // DSMEM bid-list slots per CTA
    const CLayout L = c_layout<R, IX>(N, M, CS);
    R* P = reinterpret_cast<R*>(smem + L.P);
    U* Pbits = reinterpret_cast<U*>(smem + L.P);
    int* win = reinterpret_cast<int*>(smem + L.win);
    IX* owner = reinterpret_cast<IX*>(smem + L.owner);
    IX* rowcol = reinterpret_cast<IX*>(smem + L.rowcol);
    IX* act = reinterpret_cast<IX*>(smem + L.act);
    R* lbid = reinterpret_cast<R*>(smem + L.lbid);
    IX* lrow = reinterpret_cast<IX*>(smem + L.lrow);
    IX* lcol = reinterpret_cast<IX*>(smem + L.lcol);
    Top2<R>* part = reinterpret_cast<Top2<R>*>(smem + L.part);
    int* cnt = reinterpret_cast<int*>(smem + L.cnt);
    int* evict = reinterpret_cast<int*>(smem + L.evict);
    const R tol = (R)1e-5;
    // small rounds: the slice of the columns this CTA scans (16-byte chunks)
    const int per = (nchunks + CS - 1) / CS;
    const int ch0 = rank * per, ch1 = min(nchunks, ch0 + per);
    const bool small_ok = (M >= 1024);
    // global memory of this team (only used when TC > 1)
    int* abort_flag = reinterpret_cast<int*>(p.ws);
    unsigned char* tb = p.ws + ELA_WS_HEADER + (size_t)team * p.team_bytes;
    R* pbuf = reinterpret_cast<R*>(tb + 2 * (size_t)ST * p.seg_bytes);
    unsigned int* pflag = reinterpret_cast<unsigned int*>(tb + 2 * (size_t)ST * p.seg_bytes + align_up(sizeof(R) * (size_t)M, 256));

    bool cl_pending = false;      // a "consumed" arrival on the cluster barrier awaits its wait
    unsigned int t = 0;           // global-exchange round tag (large rounds, TC > 1)
    unsigned int seq = 0;         // epsilons the leader has published (TC > 1)
    unsigned int sr = 0;          // small rounds run by this cluster (parity of the partial buffers)
    if (tid == 0) {
        s_ties = 0;
        s_exact = 0;
        s_abort = 0;
        mbar_init(&s_mbar[0], 1);
        mbar_init(&s_mbar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    cluster.sync();               // every CTA of the cluster runs before any remote store

    // ---- failure exit, taken by the whole cluster together.  A CTA leaves
    // only through a cluster barrier phase that every other resident CTA must
    // also arrive at, so until it arrives every peer is still resident: a CTA
    // that fails by itself first marks s_abort in every CTA of the cluster
    // (distributed shared memory), then arrives and waits.  Every CTA checks
    // its own s_abort after each cluster barrier wait of the round loop (a
    // failing peer's mark is released before its arrival) and then leaves the
    // same way without storing to peers, since a failed peer may have exited.
    // Waits count only resident CTAs, so the last leavers do not block.
#define ELA_CLUSTER_LEAVE() do { cluster_leave(abort_flag, cl_pending, &s_abort, CS); return; } while (0)
    // (read once per CTA: every thread of the CTA must take the same way)
#define ELA_CLUSTER_ABORT_CHECK() do { if (__syncthreads_or(*(volatile int*)&s_abort)) ELA_CLUSTER_LEAVE(); } while (0)

#ifdef ELA_PROF
    if (blockIdx.x == 0 && threadIdx.x == 0) { g_trace[8191][0] = clock64(); g_trace[8191][1] = globaltimer_ns(); }
#endif
    for (int64_t b = team; b < p.B; b += p.ngroups) {
        const In* base = reinterpret_cast<const In*>(p.cost) + b * p.stride_b;
        for (int j = tid; j < M; j += blockDim.x) { P[j] = (R)0; win[j] = 0; owner[j] = (IX)-1; }
        for (int i = tid; i < N; i += blockDim.x) rowcol[i] = (IX)-1;
        long long rounds = 0, rowbids = 0;
        int ph = 0, it = 0;
        R eps = (R)p.eps[0];  // this epsilon (read once per epsilon)
        __syncthreads();
        int K = compact_unassigned<IX, ELA_ONEPASS_COMPACT(In)>(rowcol, N, act, s_scan);  // rows that bid this round, ascending
        bool small = small_ok && K <= ELA_SMALL_ROUND;
#ifdef ELA_PROF
        long long lastS5 = 0;
#endif
        while (ph < p.n_eps) {
            if (it == p.max_iter || K == 0) {  // this epsilon is done
                PROF_MARK(E0);
                if (small) {  // the cluster's next stores into its CTAs' bid lists wait for everyone
                    if (cl_pending) { cluster_wait_acquire(); cl_pending = false; ELA_CLUSTER_ABORT_CHECK(); }
                    cluster_arrive_release();
                    cluster_wait_acquire();
                    ELA_CLUSTER_ABORT_CHECK();
                }
                if (small && TC > 1) {
                    // the leader publishes its prices; the other clusters wait for them
                    ++seq;
                    if (leader) {
                        if (rank == 0) {
                            for (int j = tid; j < M; j += blockDim.x) __stcg(pbuf + j, P[j]);
                            __threadfence();
                            __syncthreads();
                            if (tid == 0) st_release_u32(pflag, seq);
                        }
                    } else {
                        if (tid == 0) {
                            const unsigned long long t0 = globaltimer_ns();
                            int ok = 1;
                            unsigned int spins = 0;
                            while (ld_acquire_u32(pflag) < seq) {
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
                            s_fail = !ok;
                        }
                        __syncthreads();
                        if (s_fail) ELA_CLUSTER_LEAVE();
                        for (int j = tid; j < M; j += blockDim.x) P[j] = __ldcg(pbuf + j);
                    }
                }
                if (++ph >= p.n_eps) break;
                eps = (R)p.eps[ph];
                it = 0;
                for (int j = tid; j < M; j += blockDim.x) owner[j] = (IX)-1;
                for (int i = tid; i < N; i += blockDim.x) rowcol[i] = (IX)-1;
                __syncthreads();
                K = compact_unassigned<IX, ELA_ONEPASS_COMPACT(In)>(rowcol, N, act, s_scan);
                small = small_ok && K <= ELA_SMALL_ROUND;
#ifdef ELA_PROF
                if (b == 0 && leader && rank == 0 && tid == 0) {
                    atomicAdd(&g_prof[13], (unsigned long long)(clock64() - E0)); atomicAdd(&g_prof[14], 1ull);
                }
#endif
                continue;
            }
            if (small) {
                if (!leader) { K = 0; continue; }  // wait at the end of the epsilon
                PROF_MARK(S0);
#ifdef ELA_PROF
                if (b == 0 && rank == 0 && tid == 0 && lastS5) atomicAdd(&g_prof[12], (unsigned long long)(S0 - lastS5));
#endif
                if (cl_pending) {  // last round's data read everywhere
                    cluster_wait_acquire();
                    cl_pending = false;
                    ELA_CLUSTER_ABORT_CHECK();
                }
                const int bp = ASYNC ? (int)(sr & 1) : 0;
                Top2<R>* pb = part + (size_t)bp * CS * ELA_SMALL_ROUND;
                if (ASYNC && tid == 0)
                    mbar_expect_tx(&s_mbar[bp], (unsigned int)(K * (CS - 1) * sizeof(Top2<R>)));
                // ---- partial top-2 of my column slice for each active row,
                //      stored straight into every CTA of the cluster (lane d -> CTA d)
                for (int k = warp; k < K; k += nw) {
                    const In* row = base + (int64_t)act[k] * p.stride_n;
                    const uint4* rv = reinterpret_cast<const uint4*>(row);
                    Top2<R> tt;
                    top2_init(tt);
                    // the lane's chunks of the slice, loaded two at a time
                    if (ELA_EXACT16 >= 2 && sizeof(In) == 2) {
                        scan_chunks<In, R, 2, false>(rv, P, ch0 + lane, 32, ch1, tt);
                        tt = top2_warp(tt);
                    } else {
                        scan_chunks_fast<In, R, 2>(rv, P, ch0 + lane, 32, ch1, tt);
                        tt = top2_warp_fast(tt);
                    }
                    if (!(ELA_EXACT16 >= 2 && sizeof(In) == 2) && tt.p1 >= 0 && tt.v1 == tt.v2) {  // tied maximum in the slice: exact columns
                        top2_init(tt);
                        scan_chunks<In, R, 2, false>(rv, P, ch0 + lane, 32, ch1, tt);
                        tt = top2_warp(tt);
                    }
                    if (ASYNC) {
                        Top2<R>* slot = pb + rank * ELA_SMALL_ROUND + k;
                        if (lane == rank) *slot = tt;
                        else if (lane < CS)
                            st_async_16(cluster_map(smem_addr(slot), lane), *reinterpret_cast<const uint4*>(&tt),
                                        cluster_map(smem_addr(&s_mbar[bp]), lane));
                    } else if (lane < CS) {
                        cluster.map_shared_rank(pb, lane)[rank * ELA_SMALL_ROUND + k] = tt;
                    }
                }
                PROF_MARK(S1);
                if (ASYNC) {
                    if (tid == 0) s_fail = !mbar_wait(&s_mbar[bp], (sr >> 1) & 1u, p.wait_ns, &s_abort);
                    __syncthreads();
                    if (s_fail) {
                        if (tid == 0 && !*(volatile int*)&s_abort) atomicCAS(p.status, ELA_OK, ELA_ERR_TIMEOUT);
                        ELA_CLUSTER_LEAVE();
                    }
                    ++sr;
                } else {
                    cluster_arrive_release();
                    cluster_wait_acquire();
                    ELA_CLUSTER_ABORT_CHECK();
                }
                PROF_MARK(S2);
                // ---- each row's CS partials merged by one warp: column and bid
                for (int k = warp; k < K; k += nw) {
                    Top2<R> tt;
                    top2_init(tt);
                    if (lane < CS) tt = pb[lane * ELA_SMALL_ROUND + k];
                    tt = top2_warp(tt);
                    if (lane == 0) {
                        const int j1 = (tt.p2 >= 0 && !(tt.p1 == 0 && tt.p2 == 1)) ? tt.p2 : tt.p1;
                        lbid[k] = add_rn(P[j1], add_rn(sub_rn(tt.v1, tt.v2), eps));
                        lrow[k] = act[k];
                        lcol[k] = (IX)j1;
                    }
                }
                __syncthreads();
                if (!ASYNC) { cluster_arrive_release(); cl_pending = true; }  // the partials are consumed
                PROF_MARK(S3);
                rounds++;
                rowbids += K;
                // ---- election (identical in every CTA of the cluster):
                //      new price = max bid (never below the old price), in place.
                //      Up to 32 bids: entry e is thread e of warp 0, so warp
                //      barriers order the steps and the next bidders are listed
                //      in the same pass; more bids use the whole CTA.
                if (K <= 32) {
                    if (warp == 0) {
                        const bool valid = lane < K;
                        const int j = valid ? (int)lcol[lane] : 0;
                        if (valid) atomicMax(&Pbits[j], BT::to(lbid[lane]));
                        __syncwarp();
                        if (valid && absval(sub_rn(lbid[lane], P[j])) < tol) atomicMax(&win[j], win_key((int)lrow[lane], N, p.tie_rule));
                        __syncwarp();
                        int nxt = -1;  // this entry's bidder in the next round
                        if (valid) {
                            const int i = lrow[lane];
                            nxt = i;  // lost: bids again
                            if (win[j] == win_key(i, N, p.tie_rule)) {
                                const int prev = owner[j];
                                if (prev >= 0) rowcol[prev] = (IX)-1;
                                owner[j] = (IX)i;
                                rowcol[i] = (IX)j;
                                nxt = prev;  // -1: took a free column
                            }
                        }
                        __syncwarp();  // every win[] read before it is cleared
                        if (valid) win[j] = 0;
                        const unsigned m = __ballot_sync(0xffffffffu, nxt >= 0);
                        if (nxt >= 0) act[__popc(m & ((1u << lane) - 1))] = (IX)nxt;
                        if (lane == 0) s_cnt = __popc(m);
                    }
                } else {
                    for (int e = tid; e < K; e += blockDim.x) atomicMax(&Pbits[lcol[e]], BT::to(lbid[e]));
                    __syncthreads();
                    for (int e = tid; e < K; e += blockDim.x) {
                        const int j = lcol[e];
                        if (absval(sub_rn(lbid[e], P[j])) < tol) atomicMax(&win[j], win_key((int)lrow[e], N, p.tie_rule));
                    }
                    __syncthreads();
                    for (int e = tid; e < K; e += blockDim.x) {
                        const int j = lcol[e], i = lrow[e];
                        int ev = -2;
                        if (win[j] == win_key(i, N, p.tie_rule)) {
                            const int prev = owner[j];
                            if (prev >= 0) rowcol[prev] = (IX)-1;
                            owner[j] = (IX)i;
                            rowcol[i] = (IX)j;
                            ev = prev;
                        }
                        evict[e] = ev;
                    }
                    __syncthreads();
                    for (int e = tid; e < K; e += blockDim.x) win[lcol[e]] = 0;
                    // ---- next round: losers, and rows evicted by winners, in entry order
                    if (warp == 0) {
                        int pos = 0;
                        for (int e0 = 0; e0 < K; e0 += 32) {
                            const int e = e0 + lane;
                            int r = -1;
                            if (e < K) r = (evict[e] == -2) ? (int)lrow[e] : evict[e];
                            const unsigned m = __ballot_sync(0xffffffffu, r >= 0);
                            if (r >= 0) act[pos + __popc(m & ((1u << lane) - 1))] = (IX)r;
                            pos += __popc(m);
                        }
                        if (lane == 0) s_cnt = pos;
                    }
                }
                PROF_MARK(S4);
                __syncthreads();
                PROF_MARK(S5);
#ifdef ELA_PROF
                if (b == 0 && rank == 0 && tid == 0) {
                    atomicAdd(&g_prof[0], (unsigned long long)(S1 - S0)); atomicAdd(&g_prof[1], (unsigned long long)(S2 - S1));
                    atomicAdd(&g_prof[2], (unsigned long long)(S3 - S2)); atomicAdd(&g_prof[3], (unsigned long long)(S4 - S3));
                    atomicAdd(&g_prof[5], (unsigned long long)(S5 - S4)); atomicAdd(&g_prof[4], 1ull);
                }
                lastS5 = clock64();
#endif
                K = s_cnt;
                ++it;
                continue;
            }
            // ================= large round: the K active rows (ascending in act[])
            //                   dealt round-robin over the team's CTAs
            PROF_MARK(L0);
            if (tid == 0) { s_total = 0; s_extra = 0; s_fail = 0; }
            const int Kl = (K > gi) ? (K - 1 - gi) / ST + 1 : 0;  // rows gi, gi+ST, ... of act[]
            const unsigned int t1 = t + 1;
            unsigned long long* myseg =
                reinterpret_cast<unsigned long long*>(tb + (size_t)((t & 1) * ST + gi) * p.seg_bytes);
            const int wprl = (ELA_SPLIT_LARGE && sizeof(In) == 2 && Kl > 0 && 2 * Kl <= nw) ? nw / Kl : 1;
            if (wprl > 1) {
                // few rows: each row's chunks dealt to wprl warps, the exact
                // partials merged in shared memory (no small-round data is in
                // flight in a large round, so the partial buffer is free)
                if (warp < Kl * wprl)
                    large_share<In, R, IX>(plain_geo(p), p.stride_n, base, act + gi, ST, wprl,
                                           s_exact || (ELA_EXACT16 >= 1 && sizeof(In) == 2), P, part);
                __syncthreads();
            }
            for (int k = warp; k < Kl && wprl > 1; k += nw) {  // row k from its wprl partials
                const int i = act[gi + k * ST];
                Top2<R> tt;
                top2_init(tt);
                if (lane < wprl) tt = part[k * wprl + lane];
                tt = top2_warp(tt);
                if (lane == 0 && tt.v1 == tt.v2) atomicAdd(&s_ties, 1);
                int j1;
                R bid;
                finish_bid<In, R>(plain_geo(p), base + (int64_t)i * p.stride_n, P, tt, eps, lane, nullptr, nullptr, j1,
                                  bid);
                if (lane == 0) {
                    if (TC == 1) { const int slot = rank * rpc + k; lbid[slot] = bid; lrow[slot] = (IX)i; lcol[slot] = (IX)j1; }
                    else put_entry<R>(myseg, k, t1, i, j1, bid);
                }
            }
            for (int k = warp; k < Kl && wprl == 1; k += nw) {  // one warp per row
                const int i = act[gi + k * ST];
                const In* row = base + (int64_t)i * p.stride_n;
                Top2<R> tt;
                // tie-heavy rows, and 16-bit costs (whose 8-wide fast chunk costs
                // more than the exact one's filter), take one exact pass
                if (s_exact || (ELA_EXACT16 >= 1 && sizeof(In) == 2)) {
                    tt = scan_row_plain<In, R>(p, row, P, lane, 0, 1);
                } else {
                    tt = scan_row_fast<In, R>(plain_geo(p), row, P, lane, 0, 1);
                    if (tt.v1 == tt.v2) tt = scan_row_plain<In, R>(p, row, P, lane, 0, 1);
                }
                if (lane == 0 && tt.v1 == tt.v2) atomicAdd(&s_ties, 1);
                int j1;
                R bid;
                finish_bid<In, R>(plain_geo(p), row, P, tt, eps, lane, nullptr, nullptr, j1, bid);
                if (lane == 0) {
                    if (TC == 1) { const int slot = rank * rpc + k; lbid[slot] = bid; lrow[slot] = (IX)i; lcol[slot] = (IX)j1; }
                    else put_entry<R>(myseg, k, t1, i, j1, bid);
                }
            }
            __syncthreads();
            PROF_MARK(L1);
            if (tid == 0) { s_exact = (Kl > 0) ? (s_ties * 4 > Kl) : s_exact; s_ties = 0; }
            int nent;
            bool compact;  // entries at 0..nent-1 (else slots rank*rpc + k)
            if (TC == 1) {
                // ---- exchange through distributed shared memory
                if (cl_pending) { cluster_wait_acquire(); cl_pending = false; ELA_CLUSTER_ABORT_CHECK(); }
                __syncthreads();
                for (int e = tid; e < Kl * CS; e += blockDim.x) {
                    const int k = e / CS, dst = e % CS;
                    if (dst == rank) continue;
                    const int slot = rank * rpc + k;
                    cluster.map_shared_rank(lbid, dst)[slot] = lbid[slot];
                    cluster.map_shared_rank(lrow, dst)[slot] = lrow[slot];
                    cluster.map_shared_rank(lcol, dst)[slot] = lcol[slot];
                }
                if (tid < CS) cluster.map_shared_rank(cnt, tid)[rank] = Kl;
                cluster_arrive_release();
                cluster_wait_acquire();
                ELA_CLUSTER_ABORT_CHECK();
                if (tid == 0) {
                    int acc = 0;
                    for (int r = 0; r < CS; ++r) { s_off[r] = acc; acc += cnt[r]; }
                    s_off[CS] = acc;
                }
                __syncthreads();
                nent = s_off[CS];
                compact = false;
            } else {
                // ---- exchange through tagged words in global memory (every
                //      word carries the tag; readers re-read stale words)
                if (tid == 0 && !(p.skip_publish && t == 0 && gi == 0))  // (test hook: CTA 0 withholds round 0)
                    st_relaxed_u64(myseg, ((unsigned long long)t1 << 32) | (unsigned int)Kl);
                if (tid < ST) {
                    const unsigned long long* seg =
                        reinterpret_cast<const unsigned long long*>(tb + (size_t)((t & 1) * ST + tid) * p.seg_bytes);
                    const unsigned long long t0 = globaltimer_ns();
                    unsigned int spins = 0;
                    int cntv = -1;
                    constexpr int NW = 1 + Ex<R>::INL * Ex<R>::EW;
                    unsigned long long w[NW];
                    for (;;) {
#pragma unroll
                        for (int k = 0; k < NW; ++k) w[k] = ld_relaxed_u64(seg + k);
                        if ((unsigned int)(w[0] >> 32) == t1) {
                            const int cn = (int)(unsigned int)(w[0] & 0xffffffffull);
                            bool ok = true;
#pragma unroll
                            for (int k = 0; k < Ex<R>::INL; ++k)
                                if (k < cn) ok = ok && entry_tags_ok<R>(w + 1 + Ex<R>::EW * k, t1);
                            if (ok) { cntv = cn; break; }
                        }
                        if ((++spins & 15u) == 0) {
                            if (*(volatile int*)abort_flag) break;
                            if (globaltimer_ns() - t0 > p.wait_ns) {
                                atomicExch(abort_flag, 1);
                                atomicCAS(p.status, ELA_OK, ELA_ERR_TIMEOUT);
                                break;
                            }
                        }
                    }
                    if (cntv < 0) {
                        s_fail = 1;
                    } else {
                        const int off = atomicAdd(&s_total, cntv);
                        s_segcnt[tid] = cntv;
                        s_off[tid] = off;
                        if (cntv > Ex<R>::INL) s_extra = 1;
#pragma unroll
                        for (int k = 0; k < Ex<R>::INL; ++k)
                            if (k < cntv) {
                                int rr, cc;
                                R bb;
                                decode_entry<R>(w + 1 + Ex<R>::EW * k, rr, cc, bb);
                                lbid[off + k] = bb; lrow[off + k] = (IX)rr; lcol[off + k] = (IX)cc;
                            }
                    }
                }
                __syncthreads();
                if (s_fail) ELA_CLUSTER_LEAVE();
                if (s_extra && !read_extra_entries<R, IX>(tb + (size_t)((t & 1) * ST) * p.seg_bytes, p.seg_bytes, ST,
                                                          s_segcnt, s_off, s_exoff, t1, lbid, lrow, lcol, abort_flag,
                                                          p.status))
                    ELA_CLUSTER_LEAVE();
                nent = s_total;
                compact = true;
                ++t;
            }
            PROF_MARK(L2);
            rounds++;
            rowbids += nent;
            // ---- election over all bids (identical in every CTA of the team)
            auto slot_of = [&](int e) -> int {
                if (compact) return e;
                int r = 0;
                while (e >= s_off[r + 1]) ++r;
                return r * rpc + (e - s_off[r]);
            };
            // the new price of a column is its max bid (bids never fall below
            // the old price), written in place
            for (int e = tid; e < nent; e += blockDim.x) {
                const int sl = slot_of(e);
                atomicMax(&Pbits[lcol[sl]], BT::to(lbid[sl]));
            }
            __syncthreads();
            for (int e = tid; e < nent; e += blockDim.x) {
                const int sl = slot_of(e);
                const int j = lcol[sl];
                if (absval(sub_rn(lbid[sl], P[j])) < tol) atomicMax(&win[j], win_key((int)lrow[sl], N, p.tie_rule));
            }
            __syncthreads();
            for (int e = tid; e < nent; e += blockDim.x) {
                const int sl = slot_of(e);
                const int j = lcol[sl], i = lrow[sl];
                if (win[j] == win_key(i, N, p.tie_rule)) {
                    const int prev = owner[j];
                    if (prev >= 0) rowcol[prev] = (IX)-1;
                    owner[j] = (IX)i;
                    rowcol[i] = (IX)j;
                }
            }
            __syncthreads();
            for (int e = tid; e < nent; e += blockDim.x) win[lcol[slot_of(e)]] = 0;
            if (TC == 1) { cluster_arrive_release(); cl_pending = true; }  // the bids are consumed
            PROF_MARK(L3);
            ++it;
            // ---- next round's bidders (ascending); few -> small rounds
            K = compact_unassigned<IX, ELA_ONEPASS_COMPACT(In)>(rowcol, N, act, s_scan);
            if (small_ok && K <= ELA_SMALL_ROUND) small = true;
            PROF_MARK(L4);
#ifdef ELA_PROF
            if (b == 0 && leader && rank == 0 && tid == 0 && nent < 513) {
                atomicAdd(&g_prof[15], (unsigned long long)(L4 - L0)); 
            }
            if (leader && rank == 0 && tid == 0 && nent >= 513) {
                atomicAdd(&g_prof[6], (unsigned long long)(L1 - L0)); atomicAdd(&g_prof[7], (unsigned long long)(L2 - L1));
                atomicAdd(&g_prof[8], (unsigned long long)(L3 - L2)); atomicAdd(&g_prof[9], (unsigned long long)(L4 - L3));
                atomicAdd(&g_prof[10], 1ull); atomicAdd(&g_prof[11], (unsigned long long)Kl);
            }
            if (b == 0 && leader && rank == 0 && tid == 0 && it - 1 < 8192) {  // per-round trace of problem 0
                g_trace[it - 1][0] = nent; g_trace[it - 1][1] = L1 - L0; g_trace[it - 1][2] = L2 - L1;
                g_trace[it - 1][3] = L3 - L2; g_trace[it - 1][4] = L4 - L3; g_trace[it - 1][5] = Kl;
                g_trace[it - 1][6] = 1;
            }
            if (b == 0 && tid == 0 && it - 1 < 8192) {  // slowest CTA of problem 0: own scan, scan + exchange
                atomicMax(&g_trace[it - 1][7], (unsigned long long)(L1 - L0));
                atomicMax(&g_trace[it - 1][8], (unsigned long long)(L2 - L0));
            }
#endif
        }
        // ---- outputs of problem b (CTA 0 of the leader cluster); every CTA of
        //      the cluster is done with this problem's shared data
        if (cl_pending) { cluster_wait_acquire(); cl_pending = false; ELA_CLUSTER_ABORT_CHECK(); }
        cluster_arrive_release();
        cluster_wait_acquire();
        ELA_CLUSTER_ABORT_CHECK();
        __syncthreads();
        if (leader && rank == 0) {
            int un = 0;
            for (int i = tid; i < N; i += blockDim.x) {
                const int a = rowcol[i];
                p.assign_out[b * p.N + i] = a;
                un += (a < 0);
            }
            R* pout = reinterpret_cast<R*>(p.prices_out) + b * p.M;
            for (int j = tid; j < M; j += blockDim.x) pout[j] = P[j];
            if (tid == 0) s_cnt = 0;
            __syncthreads();
            if (un) atomicAdd(&s_cnt, un);
            __syncthreads();
            if (tid == 0 && p.stats_out) {
                p.stats_out[4 * b + 0] = rounds;
                p.stats_out[4 * b + 1] = rowbids;
                p.stats_out[4 * b + 2] = 0;
                p.stats_out[4 * b + 3] = s_cnt;
            }
        }
        __syncthreads();
    }
#ifdef ELA_PROF
    if (blockIdx.x == 0 && threadIdx.x == 0) { g_trace[8191][2] = clock64(); g_trace[8191][3] = globaltimer_ns(); }
#endif
    cluster.sync();  // no remote store may target a CTA that has exited
#undef ELA_CLUSTER_ABORT_CHECK
#undef ELA_CLUSTER_LEAVE
}

// ------------------------------------------------------- the bid pass alone
// One round's bids of every unassigned row against given prices, as one
// streaming pass over the cost rows: the reference's compute_bids
// (src/csrc/interface.cpp:31-40 -> launch_bid_kernel_cuda,
// src/csrc/kernels.cu:420-445) with the torch backend's column choice
// (torch_backend.py:65-88).  HBM-bound: each row is read once, so the kernel
// is a plain grid over every SM (two 256-thread CTAs per SM, each warp
// scanning whole rows with ELA_BID_UNROLL 16-byte loads in flight per lane).
// The problem's prices are staged in shared memory (zeros when none are
// given).  Rows whose assignment is not -1 get column -1 and increment 0, as
// in the reference.
#define ELA_BID_THREADS 256
#ifndef ELA_BID_UNROLL
#define ELA_BID_UNROLL 8
#endif

struct BidParams {
    const void* cost;
    int64_t B, N, M, stride_b, stride_n;
    const void* prices;         // B x M (R), or null: zeros
    const int64_t* assign;      // B x N, or null: every row bids
    double eps;
    void* col_out;              // B x N, int64 (public entry) or int32 (the solve's first round)
    void* inc_out;              // B x N increments (R): (v1 - v2) + eps
    int vec_ok;
    int col64;
};

template <typename In, typename R>
__global__ void __launch_bounds__(ELA_BID_THREADS, 2) bid_pass_kernel(const BidParams q) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int M = (int)q.M;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    R* Ps = reinterpret_cast<R*>(smem);
    const size_t poff = align_up(sizeof(R) * (size_t)M, 16);
    R* scr_v = reinterpret_cast<R*>(smem + poff) + warp * ELA_SMALL_M;
    int* scr_i = reinterpret_cast<int*>(smem + poff + sizeof(R) * (size_t)nw * ELA_SMALL_M) + warp * ELA_SMALL_M;
    const PlainGeo g{M, q.vec_ok};
    const R eps = (R)q.eps;
    const R* pr = reinterpret_cast<const R*>(q.prices);
    R* inc_out = reinterpret_cast<R*>(q.inc_out);
    if (pr == nullptr)
        for (int j = threadIdx.x; j < M; j += blockDim.x) Ps[j] = (R)0;
    for (int64_t b = blockIdx.y; b < q.B; b += gridDim.y) {
        if (pr != nullptr) {
            __syncthreads();  // the previous problem's rows are done with Ps
            for (int j = threadIdx.x; j < M; j += blockDim.x) Ps[j] = pr[b * q.M + j];
        }
        __syncthreads();
        const In* base = reinterpret_cast<const In*>(q.cost) + b * q.stride_b;
        for (int64_t i = (int64_t)blockIdx.x * nw + warp; i < q.N; i += (int64_t)gridDim.x * nw) {
            const int64_t o = b * q.N + i;
            int j1 = -1;
            R inc = (R)0;
            if (q.assign == nullptr || q.assign[o] == -1) {
                const In* row = base + i * q.stride_n;
                Top2<R> t;
                if (!q.vec_ok) {
                    t = scan_row_fast<In, R, NoSum, PlainGeo>(g, row, Ps, lane, 0, 1);
                    if (t.v1 == t.v2) t = scan_row<In, R, NoSum, PlainGeo>(g, row, Ps, lane, 0, 1);
                } else {
                    const uint4* rv = reinterpret_cast<const uint4*>(row);
                    const int nch = M / Elem<In>::W;
                    top2_init(t);
                    if (sizeof(In) == 2) {  // integer-like 16-bit costs tie often: one exact pass
                        scan_chunks<In, R, ELA_BID_UNROLL, false>(rv, Ps, lane, 32, nch, t);
                        t = top2_warp(t);
                    } else {
                        scan_chunks_fast<In, R, ELA_BID_UNROLL>(rv, Ps, lane, 32, nch, t);
                        t = top2_warp_fast(t);
                        if (t.v1 == t.v2) {  // tied maximum: the exact columns
                            top2_init(t);
                            scan_chunks<In, R, 4, false>(rv, Ps, lane, 32, nch, t);
                            t = top2_warp(t);
                        }
                    }
                }
                R bid;
                finish_bid<In, R, NoSum, PlainGeo>(g, row, Ps, t, eps, lane, scr_v, scr_i, j1, bid);
                inc = add_rn(sub_rn(t.v1, t.v2), eps);
            }
            if (lane == 0) {
                if (q.col64) reinterpret_cast<int64_t*>(q.col_out)[o] = j1;
                else reinterpret_cast<int32_t*>(q.col_out)[o] = j1;
                inc_out[o] = inc;
            }
        }
    }
}

template <typename R>
__host__ __device__ inline size_t bid_pass_smem(int64_t M) {
    return align_up(sizeof(R) * (size_t)M, 16) + (sizeof(R) + sizeof(int)) * (size_t)(ELA_BID_THREADS / 32) * ELA_SMALL_M;
}

#include "ela_implicit.cuh"

}  // namespace

// ================================================================ host side
namespace {

unsigned long long g_wait_ns = 2000000000ull;
int g_skip_publish = 0;

struct Plan {
    int path;          // ELA_PATH_CTA / GRID / CLUSTER
    int cs, nclusters; // cluster path: cluster size, clusters launched
    int team;          // cluster path: clusters per problem
    int idx16;         // cluster path: 16-bit row/column indices in shared memory
    size_t team_bytes; // cluster path: workspace per team
    int S, ngroups, rpc;
    size_t smem;       // dynamic shared memory per CTA
    size_t seg_bytes;  // S > 1
    size_t ws_bytes;   // total workspace
    int cache_k;       // one-CTA path: row-cache entries per row
    int one_threads;   // one-CTA path: threads per CTA (256: two CTAs per SM; 512: one)
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

// CTAs per problem on the multi-CTA path: all SMs shared evenly by the
// problems in flight, optionally capped by ELA_CTAS_PER_PROBLEM (tuning knob).
int ctas_per_problem(int64_t B, int64_t N, int sms, int& ngroups) {
    ngroups = (int)(B < sms ? B : sms);
    if (ngroups < 1) ngroups = 1;
    int S = sms / ngroups;
    if (const char* env = getenv("ELA_CTAS_PER_PROBLEM")) {
        const int cap = atoi(env);
        if (cap >= 2 && cap < S) S = cap;
    }
    if (S > ELA_MAX_S) S = ELA_MAX_S;
    if (S > N) S = (int)N;
    return S < 2 ? 2 : S;
}

// Clusters of `cs` CTAs of auction_cluster_kernel<R,R,IX> that fit at once with
// `smem` bytes per CTA (0 if the size is refused).
template <typename R, typename IX>
int cluster_fit(int cs, size_t smem) {
    auto kern = auction_cluster_kernel<R, R, IX>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(cs); cfg.blockDim = dim3(ELA_THREADS_CLUSTER); cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr; cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (void*)kern, &cfg) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

// Row-cache entries per row on the one-CTA path: the most (64, 60, ..., 16;
// at most 32 for up to 256 rows, where a larger cache costs more to fill
// than it saves)
// whose shared memory still lets ELA_MINB_ONE CTAs share an SM, for fp32
// prices and rows of 128..1024 columns that are whole 16-byte chunks per lane;
// 0 (no cache) otherwise.  ELA_ROW_CACHE=0 turns it off (tuning knob).
template <typename R>
int row_cache_k(int64_t N, int64_t M, int es, size_t smem_cta, int warps) {
    if (!std::is_same<R, float>::value || es == 0) return 0;
    if (const char* env = getenv("ELA_ROW_CACHE"))
        if (atoi(env) == 0) return 0;
    const int64_t per_lane = 32 * (16 / es);  // columns per 16-byte chunk slot of a warp
    if (M < ELA_SMALL_M || M % per_lane != 0 || M / per_lane > 8 || M > 65535) return 0;
    for (int kc = (N > 256 ? 64 : 32); kc >= 16; kc -= 4)
        if (k_layout<R>(N, M, (int)N, warps, kc).total <= smem_cta) return kc;
    return 0;
}

template <typename R>
int make_plan_t(int64_t B, int64_t N, int64_t M, int path, int sms, size_t smem_max, size_t smem_sm, int es,
                Plan& pl) {
    // one CTA per problem: up to twice as many problems as SMs, one CTA of 512
    // threads per SM (twice the warps for the wide early rounds, the whole SM's
    // shared memory for the row cache), the hardware starting the next problem
    // on whichever SM finishes first; larger batches, 256 threads and two CTAs
    // per SM (measured on 512^2 batches: wide 0.76 against 0.83 ms at B = 256,
    // 0.80 against 0.83 at 296; narrow ahead at 444 and 1024)
    bool wide = B <= 2 * (int64_t)sms;
    if (const char* env = getenv("ELA_WIDE_CTA")) {  // tuning knob (0: never, 2: always)
        if (atoi(env) == 0) wide = false;
        if (atoi(env) == 2) wide = true;
    }
    const int one_threads = wide ? ELA_THREADS_MULTI : ELA_THREADS_ONE;
    const int kc = row_cache_k<R>(N, M, es, wide ? smem_max : smem_sm / ELA_MINB_ONE - 1024 - 3 * 1024,
                                  one_threads / 32);
    const size_t one_smem = k_layout<R>(N, M, (int)N, one_threads / 32, kc).total;
    const bool one_fits = one_smem <= smem_max;
    int ngroups = 1;
    const int S = ctas_per_problem(B, N, sms, ngroups);
    const int rpc = (int)((N + S - 1) / S);
    const size_t multi_smem = k_layout<R>(N, M, rpc, ELA_THREADS_MULTI / 32).total;
    const bool multi_fits = multi_smem <= smem_max && N < (1 << 24) && M < (1 << 24) && N >= 2;

    // cluster plan: 16-CTA clusters when every problem gets one at once, else
    // 8-CTA clusters (more of them fit); 16-bit indices below 32768 rows/columns
    int cs = 0, max_clusters = 0;
    size_t cl_smem = 0;
    bool cl_fits = false;
    const bool idx16 = N < 32768 && M < 32768;
    const bool no_cluster = (path == -1);
    if (no_cluster) path = ELA_PATH_AUTO;
    if (!no_cluster && M >= ELA_SMALL_M && N >= 2 && N < (1 << 24) &&
        (path == ELA_PATH_AUTO || path == ELA_PATH_CLUSTER)) {
        // the largest cluster size that keeps at least 3/4 of the SMs busy
        // that the best size would (teams of clusters per problem): large
        // clusters make small rounds faster, more SMs make large rounds faster
        int force = 0;
        if (const char* env = getenv("ELA_CLUSTER_SIZE")) force = atoi(env);  // tuning knob
        int csz[4], ncl[4];
        size_t smz[4];
        long used[4], best_used = 0;
        int nc = 0;
        for (int c : {16, 8, 4, 2}) {
            if (force && c != force) continue;
            const size_t sm = idx16 ? c_layout<R, short>(N, M, c).total : c_layout<R, int>(N, M, c).total;
            if (sm > smem_max) continue;
            const int n = idx16 ? cluster_fit<R, short>(c, sm) : cluster_fit<R, int>(c, sm);
            if (n <= 0) continue;
            const long teams = B < n ? B : n;
            const long team = (B < n) ? n / B : 1;
            const long waves = (B + teams - 1) / teams;
            csz[nc] = c; ncl[nc] = n; smz[nc] = sm; used[nc] = B * team * c / waves;  // busy SMs per wave
            if (used[nc] > best_used) best_used = used[nc];
            ++nc;
        }
        for (int k = 0; k < nc; ++k)
            if (4 * used[k] >= 3 * best_used) { cs = csz[k]; max_clusters = ncl[k]; cl_smem = smz[k]; break; }
        cl_fits = cs > 0;
    }

    int chosen = path;
    if (path == ELA_PATH_AUTO) {
        if (one_fits && (N <= 512 || B >= sms)) chosen = ELA_PATH_CTA;
        else if (cl_fits) chosen = ELA_PATH_CLUSTER;
        else if (multi_fits) chosen = ELA_PATH_GRID;
        else if (one_fits) chosen = ELA_PATH_CTA;
        else return ELA_ERR_UNSUPPORTED;
    }
    pl.path = chosen;
    if (chosen == ELA_PATH_CLUSTER) {
        if (!cl_fits) return ELA_ERR_UNSUPPORTED;
        pl.cs = cs;
        pl.idx16 = idx16 ? 1 : 0;
        // few problems: a team of clusters per problem shares its large rounds
        int team = 1, nteams = max_clusters;
        if (B < max_clusters) { nteams = (int)B; team = max_clusters / (int)B; }
        if (const char* env = getenv("ELA_CLUSTERS_PER_PROBLEM")) {  // tuning knob
            const int v = atoi(env);
            if (v >= 1 && v < team) team = v;
        }
        while (team * cs > ELA_MAX_S) --team;
        pl.team = team;
        pl.ngroups = nteams;
        pl.nclusters = nteams * team;
        pl.S = team * cs;
        pl.rpc = (int)((N + pl.S - 1) / pl.S);
        pl.smem = cl_smem;
        pl.seg_bytes = align_up(8 + 8 * (size_t)Ex<R>::EW * pl.rpc, 128);
        pl.team_bytes = (team > 1) ? align_up(2 * (size_t)pl.S * pl.seg_bytes + align_up(sizeof(R) * (size_t)M, 256) + 256, 256) : 0;
        pl.ws_bytes = ELA_WS_HEADER + (size_t)nteams * pl.team_bytes;
        if (getenv("ELA_DEBUG_PLAN"))
            fprintf(stderr, "ela plan: cluster cs=%d max_clusters=%d team=%d teams=%d smem=%zu\n", cs, max_clusters,
                    team, nteams, cl_smem);
    } else if (chosen == ELA_PATH_CTA) {
        if (!one_fits) return ELA_ERR_UNSUPPORTED;
        pl.S = 1; pl.ngroups = 0; pl.rpc = (int)N;
        pl.smem = one_smem;
        pl.cache_k = kc;
        pl.one_threads = one_threads;
        pl.seg_bytes = 0;
        pl.ws_bytes = ELA_WS_HEADER;
    } else if (chosen == ELA_PATH_GRID) {
        if (!multi_fits) return ELA_ERR_UNSUPPORTED;
        pl.S = S; pl.ngroups = ngroups; pl.rpc = rpc;
        pl.smem = multi_smem;
        pl.seg_bytes = align_up(8 + 8 * (size_t)Ex<R>::EW * rpc, 128);
        pl.ws_bytes = ELA_WS_HEADER + (size_t)ngroups * 2 * S * pl.seg_bytes;
    } else {
        return ELA_ERR_ARGUMENT;
    }
    return ELA_OK;
}

int device_limits(int& sms, size_t& smem_max, size_t& smem_sm) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ELA_ERR_CUDA;
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return ELA_ERR_CUDA;
    sms = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return ELA_ERR_CUDA;
    smem_max = (size_t)v - 3 * 1024;  // room for the kernel's static shared variables
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess) return ELA_ERR_CUDA;
    smem_sm = (size_t)v;
    return ELA_OK;
}

int make_plan_uncached(int dtype, int64_t B, int64_t N, int64_t M, int path, Plan& pl, bool allow_cluster) {
    if (elem_size(dtype) == 0 || B < 0 || N < 0 || M < 0) return ELA_ERR_ARGUMENT;
    if (path < ELA_PATH_AUTO || path > ELA_PATH_CLUSTER) return ELA_ERR_ARGUMENT;
    if (N > 0 && M < 2) return ELA_ERR_ARGUMENT;
    if (N >= (1ll << 30) || M >= (1ll << 30)) return ELA_ERR_UNSUPPORTED;
    int sms = 0;
    size_t smem_max = 0, smem_sm = 0;
    const int rc = device_limits(sms, smem_max, smem_sm);
    if (rc != ELA_OK) return rc;
    if (!allow_cluster && path == ELA_PATH_CLUSTER) return ELA_ERR_UNSUPPORTED;
    const int ask = (!allow_cluster && path == ELA_PATH_AUTO) ? -1 : path;
    const int es = elem_size(dtype);
    return dtype == ELA_DTYPE_F64 ? make_plan_t<double>(B, N, M, ask, sms, smem_max, smem_sm, es, pl)
                                  : make_plan_t<float>(B, N, M, ask, sms, smem_max, smem_sm, es, pl);
}

// Plans are cached per device, sizes, path and tuning-knob settings: planning
// runs occupancy queries (several CUDA calls), which would otherwise cost more
// host time per solve than a small problem's whole solve on the GPU.
std::mutex g_plan_mu;
std::unordered_map<std::string, Plan> g_plans;

int make_plan(int dtype, int64_t B, int64_t N, int64_t M, int path, Plan& pl, bool allow_cluster = true) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ELA_ERR_CUDA;
    char key[256];
    auto knob = [](const char* name) { const char* v = getenv(name); return v ? v : "-"; };
    snprintf(key, sizeof key, "%d|%d|%lld|%lld|%lld|%d|%d|%.16s|%.16s|%.16s|%.16s", dev, dtype, (long long)B,
             (long long)N, (long long)M, path, allow_cluster ? 1 : 0, knob("ELA_CTAS_PER_PROBLEM"),
             knob("ELA_CLUSTER_SIZE"), knob("ELA_CLUSTERS_PER_PROBLEM"), knob("ELA_ROW_CACHE"));
    strncat(key, knob("ELA_WIDE_CTA"), sizeof key - strlen(key) - 1);
    {
        std::lock_guard<std::mutex> lock(g_plan_mu);
        auto it = g_plans.find(key);
        if (it != g_plans.end()) { pl = it->second; return ELA_OK; }
    }
    const int rc = make_plan_uncached(dtype, B, N, M, path, pl, allow_cluster);
    if (rc == ELA_OK) {
        std::lock_guard<std::mutex> lock(g_plan_mu);
        if (g_plans.size() >= 4096) g_plans.clear();
        g_plans.emplace(key, pl);
    }
    return rc;
}

template <typename In, typename R>
int launch_bid_pass(const BidParams& q, int ctas, cudaStream_t stream) {
    const size_t bsm = bid_pass_smem<R>(q.M);
    if (cudaFuncSetAttribute(bid_pass_kernel<In, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsm) !=
        cudaSuccess)
        return ELA_ERR_CUDA;
    const int64_t gy = q.B < 65535 ? q.B : 65535;
    const int64_t rows_x = (q.N + ELA_BID_THREADS / 32 - 1) / (ELA_BID_THREADS / 32);
    int64_t gx = (ctas + gy - 1) / gy;
    if (gx > rows_x) gx = rows_x;
    if (gx < 1) gx = 1;
    bid_pass_kernel<In, R><<<dim3((unsigned int)gx, (unsigned int)gy), ELA_BID_THREADS, bsm, stream>>>(q);
    return cudaGetLastError() == cudaSuccess ? ELA_OK : ELA_ERR_CUDA;
}

template <typename In, typename R>
int launch(const Params& p, const Plan& pl, cudaStream_t stream) {
    if (pl.path == ELA_PATH_CLUSTER) {
        if (!p.vec_ok || p.gsum || p.vpad) return ELA_ERR_UNSUPPORTED;  // 16-byte rows of one tensor
        auto kern = pl.idx16 ? auction_cluster_kernel<In, R, short> : auction_cluster_kernel<In, R, int>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess)
            return ELA_ERR_CUDA;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
            return ELA_ERR_CUDA;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = pl.cs; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeCooperative;
        attr[1].val.cooperative = 1;
        cfg.gridDim = dim3(pl.cs * pl.nclusters);
        cfg.blockDim = dim3(ELA_THREADS_CLUSTER);
        cfg.dynamicSmemBytes = pl.smem;
        cfg.stream = stream;
        cfg.attrs = attr;
        // The clusters of a team wait on one another (bounded waits), so they
        // must be resident at once.  The launch never exceeds the clusters the
        // occupancy query says fit, but other work on the GPU can hold SMs: a
        // cooperative launch makes the driver refuse a grid it cannot
        // co-schedule, and a refused team plan falls back to one cluster per
        // problem (no inter-cluster waits; same results).
        cfg.numAttrs = pl.team > 1 ? 2 : 1;
        if (const char* env = getenv("ELA_TEAM_COOPERATIVE"))  // tuning knob (A/B of the co-scheduling guarantee)
            if (atoi(env) == 0) cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
        if (e != cudaSuccess && pl.team > 1) {
            cudaGetLastError();  // the refused launch left no work behind
            if (getenv("ELA_DEBUG_PLAN"))
                fprintf(stderr, "ela plan: cooperative team launch refused (%s); one cluster per problem\n",
                        cudaGetErrorString(e));
            Params q = p;
            q.team = 1;
            q.team_bytes = 0;
            q.ngroups = (int)(p.B < pl.ngroups * (int64_t)pl.team ? p.B : pl.ngroups * (int64_t)pl.team);
            q.S = pl.cs;
            cfg.gridDim = dim3(pl.cs * q.ngroups);
            cfg.numAttrs = 1;
            e = cudaLaunchKernelEx(&cfg, kern, q);
        }
        return e == cudaSuccess ? ELA_OK : ELA_ERR_CUDA;
    }
    if (pl.S == 1) {
        const bool wide = pl.one_threads == ELA_THREADS_MULTI;
        typedef WithSum<In> WS;
        auto kern = wide ? auction_kernel<In, R, false, ELA_THREADS_MULTI, 1>
                         : auction_kernel<In, R, false, ELA_THREADS_ONE, ELA_MINB_ONE>;
        if (p.gsum)
            kern = wide ? auction_kernel<In, R, false, ELA_THREADS_MULTI, 1, false, WS>
                        : auction_kernel<In, R, false, ELA_THREADS_ONE, ELA_MINB_ONE, false, WS>;
        if constexpr (std::is_same<R, float>::value)
            if (p.cache_k > 0) {
                kern = wide ? auction_kernel<In, R, false, ELA_THREADS_MULTI, 1, true>
                            : auction_kernel<In, R, false, ELA_THREADS_ONE, ELA_MINB_ONE, true>;
                if (p.gsum)
                    kern = wide ? auction_kernel<In, R, false, ELA_THREADS_MULTI, 1, true, WS>
                                : auction_kernel<In, R, false, ELA_THREADS_ONE, ELA_MINB_ONE, true, WS>;
            }
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess)
            return ELA_ERR_CUDA;
        const int64_t grid = p.B < (1ll << 20) ? p.B : (1ll << 20);
        kern<<<(unsigned int)grid, pl.one_threads, pl.smem, stream>>>(p);
        return cudaGetLastError() == cudaSuccess ? ELA_OK : ELA_ERR_CUDA;
    }
    auto kern = p.gsum ? auction_kernel<In, R, true, ELA_THREADS_MULTI, ELA_MINB_MULTI, false, WithSum<In>>
                       : auction_kernel<In, R, true, ELA_THREADS_MULTI, ELA_MINB_MULTI>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess)
        return ELA_ERR_CUDA;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, ELA_THREADS_MULTI, pl.smem) != cudaSuccess)
        return ELA_ERR_CUDA;
    if (occ < 1) return ELA_ERR_UNSUPPORTED;
    // The CTAs of a group wait on one another, so all must be resident at
    // once: the cooperative launch refuses a grid that cannot be co-scheduled.
    Params pc = p;
    void* args[] = {&pc};
    const cudaError_t e = cudaLaunchCooperativeKernel((const void*)kern, dim3(pl.S * pl.ngroups),
                                                      dim3(ELA_THREADS_MULTI), args, pl.smem, stream);
    return e == cudaSuccess ? ELA_OK : ELA_ERR_CUDA;
}

// Validates the arguments common to the solve entry points and fills Params
// (everything except the workspace pointers).
int fill_params(const void* cost, int dtype, int64_t B, int64_t N, int64_t M, int64_t stride_b,
                int64_t stride_n, const double* eps_schedule, int n_eps, int max_iter, int tie_rule,
                int64_t* assign_out, void* prices_out, int64_t* stats_out, Params& p) {
    const int es = elem_size(dtype);
    if (!cost || !assign_out || !prices_out) return ELA_ERR_ARGUMENT;
    if (tie_rule != ELA_TIE_HIGHEST_ROW && tie_rule != ELA_TIE_LOWEST_ROW) return ELA_ERR_ARGUMENT;
    if (stride_n < M || (B > 1 && stride_b < (N - 1) * stride_n + M)) return ELA_ERR_ARGUMENT;
    memset(&p, 0, sizeof(p));
    p.cost = cost;
    p.B = B; p.N = N; p.M = M; p.stride_b = stride_b; p.stride_n = stride_n;
    for (int k = 0; k < n_eps; ++k) p.eps[k] = eps_schedule[k];
    p.n_eps = n_eps;
    p.max_iter = max_iter;
    p.tie_rule = tie_rule;
    p.vec_ok = ((reinterpret_cast<uintptr_t>(cost) & 15u) == 0) && ((stride_n * es) % 16 == 0) &&
               ((stride_b * es) % 16 == 0) && ((M * es) % 16 == 0);
    p.assign_out = assign_out;
    p.prices_out = prices_out;
    p.stats_out = stats_out;
    p.wait_ns = g_wait_ns;
    p.skip_publish = g_skip_publish;
    p.max_wpr = 32;
    if (const char* env = getenv("ELA_MAX_WARPS_PER_ROW")) {  // tuning knob
        const int v = atoi(env);
        if (v >= 1) p.max_wpr = v;
    }
    return ELA_OK;
}

// Argument checks that need no device; returns ELA_OK to continue, or a
// status.  *done is set when there is nothing to solve (after clearing outputs).
int check_common(int dtype, int64_t B, int64_t N, int64_t M, const double* eps_schedule, int n_eps,
                 int max_iter, void* prices_out, int64_t* stats_out, int32_t* status_out,
                 cudaStream_t s, bool* done) {
    *done = false;
    if (elem_size(dtype) == 0 || B < 0 || N < 0 || M < 0 || max_iter < 0) return ELA_ERR_ARGUMENT;
    if (n_eps < 1 || n_eps > ELA_MAX_PHASES || eps_schedule == nullptr) return ELA_ERR_ARGUMENT;
    for (int k = 0; k < n_eps; ++k)
        if (!(eps_schedule[k] > 0.0) || eps_schedule[k] == INFINITY) return ELA_ERR_ARGUMENT;
    if (B == 0 || N == 0) {
        *done = true;
        if (B > 0 && M > 0 && prices_out &&
            cudaMemsetAsync(prices_out, 0, (size_t)(B * M) * (dtype == ELA_DTYPE_F64 ? 8 : 4), s) != cudaSuccess)
            return ELA_ERR_CUDA;
        if (stats_out && B > 0 && cudaMemsetAsync(stats_out, 0, (size_t)B * 32, s) != cudaSuccess)
            return ELA_ERR_CUDA;
        if (status_out && cudaMemsetAsync(status_out, 0, 4, s) != cudaSuccess) return ELA_ERR_CUDA;
    }
    return ELA_OK;
}

int dispatch(int dtype, const Params& p, const Plan& pl, cudaStream_t s) {
    switch (dtype) {
    case ELA_DTYPE_F32: return launch<float, float>(p, pl, s);
    case ELA_DTYPE_F16: return launch<__half, float>(p, pl, s);
    case ELA_DTYPE_BF16: return launch<__nv_bfloat16, float>(p, pl, s);
    default: return launch<double, double>(p, pl, s);
    }
}

// ------------------------------------------------- allocation-free variant
// Scratch for ela_auction_solve_noalloc: a fixed array in every device's global
// memory, reserved when the library is loaded and held until the process
// exits.  Host code sees only a stand-in symbol; the device address comes from
// cudaGetSymbolAddress, looked up once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[ELA_NOALLOC_SCRATCH_BYTES];

// The address is a property of the context that loaded the module: it is
// cached per (device, current context), so a context replaced by
// cudaDeviceReset (or a non-primary context made current by the caller) gets
// its own lookup instead of a stale address.  cuCtxGetCurrent is reached
// through the runtime's driver entry point, so the library does not link
// libcuda.
typedef int (*ela_ctx_get_current_fn)(void**);
std::mutex g_noalloc_mu;
struct NoallocSlot { int dev; void* ctx; void* ptr; };
#define ELA_NOALLOC_SLOTS 64
NoallocSlot g_noalloc_slots[ELA_NOALLOC_SLOTS];
int g_noalloc_used = 0;
ela_ctx_get_current_fn g_ctx_get_current = nullptr;

int noalloc_scratch(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ELA_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_ctx_get_current == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || fn == nullptr)
            return ELA_ERR_CUDA;
        g_ctx_get_current = reinterpret_cast<ela_ctx_get_current_fn>(fn);
    }
    void* ctx = nullptr;
    if (g_ctx_get_current(&ctx) != 0) return ELA_ERR_CUDA;
    if (ctx == nullptr) {  // no context current on this thread yet: the lookup makes the primary one current
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return ELA_ERR_CUDA;
        if (g_ctx_get_current(&ctx) != 0 || ctx == nullptr) return ELA_ERR_CUDA;
    }
    for (int k = 0; k < g_noalloc_used; ++k)
        if (g_noalloc_slots[k].dev == dev && g_noalloc_slots[k].ctx == ctx) { *out = g_noalloc_slots[k].ptr; return ELA_OK; }
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return ELA_ERR_CUDA;
    if (g_noalloc_used == ELA_NOALLOC_SLOTS) g_noalloc_used = 0;  // forget the oldest contexts
    g_noalloc_slots[g_noalloc_used++] = NoallocSlot{dev, ctx, ptr};
    *out = ptr;
    return ELA_OK;
}

}  // namespace

extern "C" {

int ela_auction_version(void) { return 200; }

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
    Plan pl = {};
    if (make_plan(dtype, B, N, M, path, pl) != ELA_OK) return 0;
    size_t ws = pl.ws_bytes;
    // AUTO may fall back from the cluster path for rows without 16-byte alignment
    Plan alt = {};
    if (path == ELA_PATH_AUTO && make_plan(dtype, B, N, M, path, alt, false) == ELA_OK && alt.ws_bytes > ws)
        ws = alt.ws_bytes;
    return ws;
}

void ela_auction_set_wait_limit_ns(uint64_t ns) { g_wait_ns = ns ? ns : 1; }

void ela_auction_debug_skip_arrive(int on) { g_skip_publish = on ? 1 : 0; }

int ela_auction_solve(const void* cost, int dtype, int64_t B, int64_t N, int64_t M,
                      int64_t stride_b, int64_t stride_n, const double* eps_schedule,
                      int n_eps, int max_iter, int path, int tie_rule, int64_t* assign_out,
                      void* prices_out, int64_t* stats_out, int32_t* status_out,
                      void* workspace, size_t workspace_bytes, void* stream) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    bool done = false;
    int rc = check_common(dtype, B, N, M, eps_schedule, n_eps, max_iter, prices_out, stats_out, status_out, s, &done);
    if (rc != ELA_OK || done) return rc;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return ELA_ERR_ARGUMENT;
    Params p;
    rc = fill_params(cost, dtype, B, N, M, stride_b, stride_n, eps_schedule, n_eps, max_iter, tie_rule,
                     assign_out, prices_out, stats_out, p);
    if (rc != ELA_OK) return rc;
    Plan pl = {};
    rc = make_plan(dtype, B, N, M, path, pl, p.vec_ok != 0);
    if (rc != ELA_OK) return rc;
    if (workspace_bytes < pl.ws_bytes) return ELA_ERR_ARGUMENT;
    unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
    p.status = status_out ? status_out : reinterpret_cast<int32_t*>(ws + 4);
    p.ws = ws;
    p.seg_bytes = pl.seg_bytes;
    p.S = pl.S;
    p.ngroups = pl.ngroups;
    p.rows_per_cta = pl.rpc;
    p.team = pl.team;
    p.team_bytes = pl.team_bytes;
    p.cache_k = p.vec_ok ? pl.cache_k : 0;
    if (cudaMemsetAsync(workspace, 0, pl.ws_bytes, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (status_out && cudaMemsetAsync(status_out, 0, 4, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (stats_out && cudaMemsetAsync(stats_out, 0, (size_t)B * 32, s) != cudaSuccess) return ELA_ERR_CUDA;
    return dispatch(dtype, p, pl, s);
}


// The reference's padding (pad_input, src/efficient_linear_assignment/utils.py:32-105)
// without the padded copy: the kernel solves the (B, N', M') problem and
// synthesises the padding blocks in its loaders.  See include/ela_auction.h.
int ela_auction_solve_padded(const void* cost, int dtype, int64_t B, int64_t N, int64_t M,
                             int64_t stride_b, int64_t stride_n, int multiple, const double* eps_schedule,
                             int n_eps, int max_iter, int path, int tie_rule, int64_t* assign_out,
                             void* prices_out, int64_t* stats_out, int32_t* status_out,
                             void* workspace, size_t workspace_bytes, void* stream) {
    if (multiple < 1 || N < 1 || M < 1) return ELA_ERR_ARGUMENT;
    const int64_t Np = (N + multiple - 1) / multiple * multiple, Mp = (M + multiple - 1) / multiple * multiple;
    if (Np == N && Mp == M)
        return ela_auction_solve(cost, dtype, B, N, M, stride_b, stride_n, eps_schedule, n_eps, max_iter, path,
                                 tie_rule, assign_out, prices_out, stats_out, status_out, workspace, workspace_bytes,
                                 stream);
    if (path == ELA_PATH_CLUSTER) return ELA_ERR_UNSUPPORTED;  // the cluster kernel needs 16-byte rows
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    bool done = false;
    int rc = check_common(dtype, B, Np, Mp, eps_schedule, n_eps, max_iter, prices_out, stats_out, status_out, s, &done);
    if (rc != ELA_OK || done) return rc;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return ELA_ERR_ARGUMENT;
    Params p;
    rc = fill_params(cost, dtype, B, N, M, stride_b, stride_n, eps_schedule, n_eps, max_iter, tie_rule, assign_out,
                     prices_out, stats_out, p);
    if (rc != ELA_OK) return rc;
    p.N = Np;
    p.M = Mp;
    p.Nr = N;
    p.Mr = M;
    p.vpad = 1;
    p.vec_ok = 0;  // scalar loads synthesise the padding
    // 1e9 as the input dtype holds it (fp16: +inf), as torch.full(..., 1e9, dtype) does
    double pad = 1e9;
    if (dtype == ELA_DTYPE_F32) pad = (double)(float)1e9;
    else if (dtype == ELA_DTYPE_F16) pad = (double)__half2float(__float2half_rn(1e9f));
    else if (dtype == ELA_DTYPE_BF16) pad = (double)__bfloat162float(__float2bfloat16_rn(1e9f));
    p.pad_c = pad;
    p.dd_c = (Np > N && Mp > M) ? 0.0 : pad;  // the padding-row x padding-column block is 0 only when both pad
    Plan pl = {};
    rc = make_plan(dtype, B, Np, Mp, path, pl, false);
    if (rc != ELA_OK) return rc;
    if (workspace_bytes < pl.ws_bytes) return ELA_ERR_ARGUMENT;
    unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
    p.status = status_out ? status_out : reinterpret_cast<int32_t*>(ws + 4);
    p.ws = ws;
    p.seg_bytes = pl.seg_bytes;
    p.S = pl.S;
    p.ngroups = pl.ngroups;
    p.rows_per_cta = pl.rpc;
    p.team = pl.team;
    p.team_bytes = pl.team_bytes;
    p.cache_k = 0;
    if (cudaMemsetAsync(workspace, 0, pl.ws_bytes, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (status_out && cudaMemsetAsync(status_out, 0, 4, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (stats_out && cudaMemsetAsync(stats_out, 0, (size_t)B * 32, s) != cudaSuccess) return ELA_ERR_CUDA;
    return dispatch(dtype, p, pl, s);
}

// The IMLE backward's target solve on cost + lam * grad without materialising
// the sum.  See include/ela_auction.h.
int ela_auction_solve_sum(const void* cost, const void* grad, double lam, int dtype, int64_t B, int64_t N,
                          int64_t M, int64_t stride_b, int64_t stride_n, const double* eps_schedule, int n_eps,
                          int max_iter, int path, int tie_rule, int64_t* assign_out, void* prices_out,
                          int64_t* stats_out, int32_t* status_out, void* workspace, size_t workspace_bytes,
                          void* stream) {
    if (path == ELA_PATH_CLUSTER) return ELA_ERR_UNSUPPORTED;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    bool done = false;
    int rc = check_common(dtype, B, N, M, eps_schedule, n_eps, max_iter, prices_out, stats_out, status_out, s, &done);
    if (rc != ELA_OK || done) return rc;
    if (!grad || !(lam == lam) || lam == INFINITY || lam == -INFINITY) return ELA_ERR_ARGUMENT;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return ELA_ERR_ARGUMENT;
    Params p;
    rc = fill_params(cost, dtype, B, N, M, stride_b, stride_n, eps_schedule, n_eps, max_iter, tie_rule, assign_out,
                     prices_out, stats_out, p);
    if (rc != ELA_OK) return rc;
    p.gsum = 1;
    p.gdiff = (long long)(reinterpret_cast<const char*>(grad) - reinterpret_cast<const char*>(cost));
    p.lam = lam;
    if ((reinterpret_cast<uintptr_t>(grad) & 15u) != 0) p.vec_ok = 0;
    Plan pl = {};
    rc = make_plan(dtype, B, N, M, path, pl, false);
    if (rc != ELA_OK) return rc;
    if (workspace_bytes < pl.ws_bytes) return ELA_ERR_ARGUMENT;
    unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
    p.status = status_out ? status_out : reinterpret_cast<int32_t*>(ws + 4);
    p.ws = ws;
    p.seg_bytes = pl.seg_bytes;
    p.S = pl.S;
    p.ngroups = pl.ngroups;
    p.rows_per_cta = pl.rpc;
    p.team = pl.team;
    p.team_bytes = pl.team_bytes;
    p.cache_k = p.vec_ok ? pl.cache_k : 0;
    if (cudaMemsetAsync(workspace, 0, pl.ws_bytes, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (status_out && cudaMemsetAsync(status_out, 0, 4, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (stats_out && cudaMemsetAsync(stats_out, 0, (size_t)B * 32, s) != cudaSuccess) return ELA_ERR_CUDA;
    return dispatch(dtype, p, pl, s);
}

// Implicit low-rank costs C = Q K^T on the tensor cores (ela_implicit.cuh).
static int implicit_launch(const void* Q, const void* Kf, int dtype, int64_t B, int64_t N, int64_t M, int64_t D,
                           const double* eps_schedule, int n_eps, int max_iter, int tie_rule, int64_t* assign_out,
                           float* prices_out, int64_t* stats_out, int32_t* status_out, float* cost_out,
                           void* stream) {
    if (dtype != ELA_DTYPE_BF16 && dtype != ELA_DTYPE_F16) return ELA_ERR_ARGUMENT;
    if (B < 0 || N < 1 || M < ELA_SMALL_M || M > 128 * ELA_IMP_MAX_TILES || D < 16 || D > 256 || D % 16 != 0)
        return ELA_ERR_ARGUMENT;
    if (!Q || !Kf || !status_out || (reinterpret_cast<uintptr_t>(Q) & 15u) || (reinterpret_cast<uintptr_t>(Kf) & 15u))
        return ELA_ERR_ARGUMENT;
    if (tie_rule != ELA_TIE_HIGHEST_ROW && tie_rule != ELA_TIE_LOWEST_ROW) return ELA_ERR_ARGUMENT;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    ImpParams p;
    memset(&p, 0, sizeof(p));
    p.Q = Q; p.Kf = Kf; p.half = dtype == ELA_DTYPE_F16;
    p.B = B; p.N = N; p.M = M; p.D = D;
    if (!cost_out) {
        if (n_eps < 1 || n_eps > ELA_MAX_PHASES || !eps_schedule || max_iter < 0 || !assign_out || !prices_out)
            return ELA_ERR_ARGUMENT;
        for (int k = 0; k < n_eps; ++k) {
            if (!(eps_schedule[k] > 0.0) || eps_schedule[k] == INFINITY) return ELA_ERR_ARGUMENT;
            p.eps[k] = eps_schedule[k];
        }
    }
    p.n_eps = n_eps; p.max_iter = max_iter; p.tie_rule = tie_rule;
    p.assign_out = assign_out; p.prices_out = prices_out; p.stats_out = stats_out; p.status = status_out;
    p.cost_out = cost_out;
    p.wait_ns = g_wait_ns;
    int sms = 0;
    size_t smem_max = 0, smem_sm = 0;
    int rc = device_limits(sms, smem_max, smem_sm);
    if (rc != ELA_OK) return rc;
    const size_t smem = i_layout(N, M, D).total;
    if (smem > smem_max) return ELA_ERR_UNSUPPORTED;
    if (cudaMemsetAsync(status_out, 0, 4, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (B == 0) return ELA_OK;
    if (cudaFuncSetAttribute(implicit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return ELA_ERR_CUDA;
    const int64_t grid = B < (1ll << 20) ? B : (1ll << 20);
    implicit_kernel<<<(unsigned int)grid, ELA_IMP_THREADS, smem, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? ELA_OK : ELA_ERR_CUDA;
}

int ela_auction_solve_implicit(const void* Q, const void* K, int dtype, int64_t B, int64_t N, int64_t M, int64_t D,
                               const double* eps_schedule, int n_eps, int max_iter, int tie_rule,
                               int64_t* assign_out, float* prices_out, int64_t* stats_out, int32_t* status_out,
                               void* stream) {
    return implicit_launch(Q, K, dtype, B, N, M, D, eps_schedule, n_eps, max_iter, tie_rule, assign_out, prices_out,
                           stats_out, status_out, nullptr, stream);
}

int ela_auction_implicit_costs(const void* Q, const void* K, int dtype, int64_t B, int64_t N, int64_t M, int64_t D,
                               float* cost_out, int32_t* status_out, void* stream) {
    if (!cost_out) return ELA_ERR_ARGUMENT;
    return implicit_launch(Q, K, dtype, B, N, M, D, nullptr, 0, 0, ELA_TIE_HIGHEST_ROW, nullptr, nullptr, nullptr,
                           status_out, cost_out, stream);
}

// Same solve as ela_auction_solve, with its scratch in g_noalloc_scratch
// instead of a caller-supplied workspace; see include/ela_auction.h.
int ela_auction_solve_noalloc(const void* cost, int dtype, int64_t B, int64_t N, int64_t M,
                              int64_t stride_b, int64_t stride_n, const double* eps_schedule,
                              int n_eps, int max_iter, int path, int tie_rule,
                              int64_t* assign_out, void* prices_out, int64_t* stats_out,
                              int32_t* status_out, void* stream) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    bool done = false;
    int rc = check_common(dtype, B, N, M, eps_schedule, n_eps, max_iter, prices_out, stats_out, status_out, s, &done);
    if (rc != ELA_OK || done) return rc;
    Params p;
    rc = fill_params(cost, dtype, B, N, M, stride_b, stride_n, eps_schedule, n_eps, max_iter, tie_rule,
                     assign_out, prices_out, stats_out, p);
    if (rc != ELA_OK) return rc;
    Plan pl = {};
    rc = make_plan(dtype, B, N, M, path, pl, p.vec_ok != 0);
    if (rc != ELA_OK) return rc;
    if (pl.ws_bytes > (size_t)ELA_NOALLOC_SCRATCH_BYTES) return ELA_ERR_UNSUPPORTED;
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc != ELA_OK) return rc;
    unsigned char* ws = reinterpret_cast<unsigned char*>(scratch);
    p.status = status_out ? status_out : reinterpret_cast<int32_t*>(ws + 4);
    p.ws = ws;
    p.seg_bytes = pl.seg_bytes;
    p.S = pl.S;
    p.ngroups = pl.ngroups;
    p.rows_per_cta = pl.rpc;
    p.team = pl.team;
    p.team_bytes = pl.team_bytes;
    p.cache_k = p.vec_ok ? pl.cache_k : 0;
    // The array keeps the previous call's contents: clear the part this solve
    // uses (abort flag, status word, exchange tags must start at zero).
    if (cudaMemsetAsync(scratch, 0, pl.ws_bytes, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (status_out && cudaMemsetAsync(status_out, 0, 4, s) != cudaSuccess) return ELA_ERR_CUDA;
    if (stats_out && cudaMemsetAsync(stats_out, 0, (size_t)B * 32, s) != cudaSuccess) return ELA_ERR_CUDA;
    return dispatch(dtype, p, pl, s);
}

// The bid pass alone: the reference's compute_bids (src/csrc/interface.cpp:31-40).
int ela_auction_compute_bids(const void* cost, int dtype, int64_t B, int64_t N, int64_t M, int64_t stride_b,
                             int64_t stride_n, const void* prices, const int64_t* assignment, double epsilon,
                             int64_t* best_idx_out, void* increments_out, void* stream) {
    const int es = elem_size(dtype);
    if (es == 0 || B < 0 || N < 0 || M < 0) return ELA_ERR_ARGUMENT;
    if (B == 0 || N == 0) return ELA_OK;
    if (M < 2 || M >= (1ll << 30) || !cost || !best_idx_out || !increments_out) return ELA_ERR_ARGUMENT;
    if (!(epsilon >= 0.0) || epsilon == INFINITY) return ELA_ERR_ARGUMENT;
    if (stride_n < M || (B > 1 && stride_b < (N - 1) * stride_n + M)) return ELA_ERR_ARGUMENT;
    int sms = 0;
    size_t smem_max = 0, smem_sm = 0;
    int rc = device_limits(sms, smem_max, smem_sm);
    if (rc != ELA_OK) return rc;
    const size_t bsm = (dtype == ELA_DTYPE_F64) ? bid_pass_smem<double>(M) : bid_pass_smem<float>(M);
    if (bsm > smem_max) return ELA_ERR_UNSUPPORTED;  // the problem's prices are staged in shared memory
    BidParams q = {};
    q.cost = cost;
    q.B = B; q.N = N; q.M = M; q.stride_b = stride_b; q.stride_n = stride_n;
    q.prices = prices;
    q.assign = assignment;
    q.eps = epsilon;
    q.col_out = best_idx_out;
    q.inc_out = increments_out;
    q.col64 = 1;
    q.vec_ok = ((reinterpret_cast<uintptr_t>(cost) & 15u) == 0) && ((stride_n * es) % 16 == 0) &&
               ((stride_b * es) % 16 == 0) && ((M * es) % 16 == 0);
    const void* bk = (dtype == ELA_DTYPE_F64) ? (const void*)bid_pass_kernel<double, double>
                   : (dtype == ELA_DTYPE_F16) ? (const void*)bid_pass_kernel<__half, float>
                   : (dtype == ELA_DTYPE_BF16) ? (const void*)bid_pass_kernel<__nv_bfloat16, float>
                                               : (const void*)bid_pass_kernel<float, float>;
    int occ = 0;
    if (cudaFuncSetAttribute(bk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsm) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, bk, ELA_BID_THREADS, bsm) != cudaSuccess)
        return ELA_ERR_CUDA;
    if (occ < 1) return ELA_ERR_UNSUPPORTED;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (dtype) {
    case ELA_DTYPE_F32: return launch_bid_pass<float, float>(q, occ * sms, s);
    case ELA_DTYPE_F16: return launch_bid_pass<__half, float>(q, occ * sms, s);
    case ELA_DTYPE_BF16: return launch_bid_pass<__nv_bfloat16, float>(q, occ * sms, s);
    default: return launch_bid_pass<double, double>(q, occ * sms, s);
    }
}

#ifdef ELA_PROF
void ela_prof_read(unsigned long long* out) { cudaMemcpyFromSymbol(out, g_prof, sizeof(g_prof)); }
void ela_trace_read(unsigned long long* out) { cudaMemcpyFromSymbol(out, g_trace, sizeof(g_trace)); }
void ela_prof_reset(void) { unsigned long long z[16] = {0}; cudaMemcpyToSymbol(g_prof, z, sizeof(z)); }
#endif
}  // extern "C"
