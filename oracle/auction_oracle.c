/*
 * auction_oracle.c -- CPU restatement of the reference auction solver.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA solver is
 * compared against (tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg).  The product path never calls it.
 *
 * What it restates: AuctionTorch.solve from the reference project,
 *   src/efficient_linear_assignment/auction/torch_backend.py:9-159
 * run with one torch thread (with more threads torch's index_put_ on duplicate
 * indices is racy, so only the one-thread result is well defined).
 *
 * One Jacobi round (torch_backend.py:54-156), for every problem b of the batch:
 *   1. active rows = rows with assignment -1, ascending            (:56-61)
 *   2. v[j] = (-c[i][j]) - P[j] in the price type R                 (:24,65-76)
 *      top-2 of v keeping duplicates: (v1, j1), v2                   (:81-85)
 *      inc = (v1 - v2) + (R)eps                                      (:88)
 *      bid = P[j1] + inc (P read before any update of this round)   (:93-99)
 *   3. P[j] = max(P[j], max of bids on j)   (scatter_reduce amax)    (:102)
 *   4. potential winners: |bid - P[j1]| < (R)1e-5                    (:106-109)
 *      elected winner per column = the highest row among them
 *      (index_put_ with ascending agents: last writer wins)          (:126-136)
 *   5. previous owner of a won column becomes -1, winner takes it    (:144-156)
 *   Loop ends when no row is active or after max_iter rounds         (:54,60-61)
 *
 * Types: R = float for fp32/fp16/bf16 input, double for fp64 input.  Half
 * inputs are widened to float first: the reference keeps prices in the half
 * dtype (torch_backend.py:27), but the solver under test keeps fp32 prices,
 * so the oracle for a half input is AuctionTorch.solve(cost.float()).
 *
 * Column tie rule: torch.topk(k=2) on CPU (torch_backend.py:81) copies the row
 * into (value, index) pairs and, for k*64 <= M, runs std::partial_sort with the
 * comparator "a.value > b.value"; otherwise std::nth_element (introselect) on
 * position k-1.  Both are deterministic, so which tied column wins is a fixed
 * function of the row.  topk_row() restates what those two libstdc++
 * algorithms return for k=2 (checked against torch.topk on random tie-heavy
 * rows by tests/test_oracle.py):
 *   M >= 128: let p1 < p2 be the first two columns holding the maximum V; the
 *             top-1 column is p2, except when (p1,p2) == (0,1) or V occurs
 *             once, where it is p1;
 *   M <  128: the result of the introselect steps below.
 * Rows whose maximum is tied are still counted (stats[2]) for reporting.
 *
 * epsilon schedule (n_eps > 1): not in the reference, which has one constant
 * epsilon and zero starting prices (torch_backend.py:27,88).  Phase k here is
 * a complete AuctionTorch.solve with epsilon eps[k] whose prices start from
 * phase k-1's final prices, with assignment and ownership reset to -1 and its
 * own max_iter round budget.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { ELA_F32 = 0, ELA_F16 = 1, ELA_BF16 = 2, ELA_F64 = 3 };

static float f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) & 1u, e = (uint32_t)(h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        /* zero or subnormal: value = m * 2^-24, exact in float */
        float f = ldexpf((float)m, -24);
        return s ? -f : f;
    } else if (e == 31) {
        bits = (s << 31) | 0x7f800000u | (m << 13);
    } else {
        bits = (s << 31) | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Load row i of problem b into buf[0..M) as R, negated (benefit = -cost). */
#define DEFINE_ROW_LOADER(R, NAME)                                                          \
    static void NAME(const void* cost, int dtype, int64_t off, int64_t M, R* buf) {         \
        int64_t j;                                                                          \
        switch (dtype) {                                                                    \
        case ELA_F32: { const float* p = (const float*)cost + off;                          \
            for (j = 0; j < M; ++j) buf[j] = (R)(-p[j]); } break;                           \
        case ELA_F16: { const uint16_t* p = (const uint16_t*)cost + off;                    \
            for (j = 0; j < M; ++j) buf[j] = (R)(-f16_to_f32(p[j])); } break;               \
        case ELA_BF16: { const uint16_t* p = (const uint16_t*)cost + off;                   \
            for (j = 0; j < M; ++j) buf[j] = (R)(-bf16_to_f32(p[j])); } break;              \
        default: { const double* p = (const double*)cost + off;                             \
            for (j = 0; j < M; ++j) buf[j] = (R)(-p[j]); } break;                           \
        }                                                                                   \
    }

DEFINE_ROW_LOADER(float, load_row_f)
DEFINE_ROW_LOADER(double, load_row_d)

/*
 * Top-2 of v[0..M) as torch.topk(k=2, largest=True) returns it on CPU.
 * Comparator of the reference's sort: less(a, b) := a.v > b.v.
 */
#define DEFINE_TOPK(R, NAME)                                                                \
    typedef struct { R v; int64_t i; } NAME##_pair;                                         \
    static int NAME##_less(const NAME##_pair* a, const NAME##_pair* b) { return a->v > b->v; } \
    static void NAME##_swap(NAME##_pair* a, NAME##_pair* b) { NAME##_pair t = *a; *a = *b; *b = t; } \
    /* binary heap on q[0..len) under less(); hole sift as in the published STL heap */    \
    static void NAME##_push(NAME##_pair* q, int64_t hole, int64_t top, NAME##_pair val) {  \
        int64_t parent = (hole - 1) / 2;                                                    \
        while (hole > top && NAME##_less(&q[parent], &val)) {                               \
            q[hole] = q[parent]; hole = parent; parent = (hole - 1) / 2;                    \
        }                                                                                   \
        q[hole] = val;                                                                      \
    }                                                                                       \
    static void NAME##_adjust(NAME##_pair* q, int64_t hole, int64_t len, NAME##_pair val) { \
        const int64_t top = hole; int64_t child = hole;                                     \
        while (child < (len - 1) / 2) {                                                     \
            child = 2 * (child + 1);                                                        \
            if (NAME##_less(&q[child], &q[child - 1])) child--;                             \
            q[hole] = q[child]; hole = child;                                               \
        }                                                                                   \
        if ((len & 1) == 0 && child == (len - 2) / 2) {                                     \
            child = 2 * (child + 1); q[hole] = q[child - 1]; hole = child - 1;              \
        }                                                                                   \
        NAME##_push(q, hole, top, val);                                                     \
    }                                                                                       \
    static void NAME##_make_heap(NAME##_pair* q, int64_t len) {                             \
        if (len < 2) return;                                                                \
        for (int64_t parent = (len - 2) / 2;; --parent) {                                   \
            NAME##_adjust(q, parent, len, q[parent]);                                       \
            if (parent == 0) return;                                                        \
        }                                                                                   \
    }                                                                                       \
    /* heap selection of the len smallest-under-less among q[0..n) into q[0..len) */       \
    static void NAME##_heap_select(NAME##_pair* q, int64_t len, int64_t n) {                \
        NAME##_make_heap(q, len);                                                           \
        for (int64_t i = len; i < n; ++i)                                                   \
            if (NAME##_less(&q[i], &q[0])) {                                                \
                NAME##_pair val = q[i]; q[i] = q[0]; NAME##_adjust(q, 0, len, val);         \
            }                                                                               \
    }                                                                                       \
    static void NAME##_introselect(NAME##_pair* q, int64_t first, int64_t nth, int64_t last, int depth) { \
        while (last - first > 3) {                                                          \
            if (depth == 0) {                                                               \
                NAME##_heap_select(q + first, nth + 1 - first, last - first);               \
                NAME##_swap(&q[first], &q[nth]);                                            \
                return;                                                                     \
            }                                                                               \
            --depth;                                                                        \
            int64_t mid = first + (last - first) / 2, a = first + 1, b = mid, c = last - 1, s; \
            if (NAME##_less(&q[a], &q[b])) {                                                \
                if (NAME##_less(&q[b], &q[c])) s = b;                                       \
                else if (NAME##_less(&q[a], &q[c])) s = c;                                  \
                else s = a;                                                                 \
            } else if (NAME##_less(&q[a], &q[c])) s = a;                                    \
            else if (NAME##_less(&q[b], &q[c])) s = c;                                      \
            else s = b;                                                                     \
            NAME##_swap(&q[first], &q[s]);                                                  \
            int64_t lo = first + 1, hi = last;                                              \
            for (;;) {                                                                      \
                while (NAME##_less(&q[lo], &q[first])) ++lo;                                \
                --hi;                                                                       \
                while (NAME##_less(&q[first], &q[hi])) --hi;                                \
                if (!(lo < hi)) break;                                                      \
                NAME##_swap(&q[lo], &q[hi]); ++lo;                                          \
            }                                                                               \
            if (lo <= nth) first = lo; else last = lo;                                      \
        }                                                                                   \
        for (int64_t i = first + 1; i < last; ++i) {                                        \
            NAME##_pair val = q[i];                                                         \
            if (NAME##_less(&val, &q[first])) {                                             \
                for (int64_t k = i; k > first; --k) q[k] = q[k - 1];                        \
                q[first] = val;                                                             \
            } else {                                                                        \
                int64_t k = i;                                                              \
                while (NAME##_less(&val, &q[k - 1])) { q[k] = q[k - 1]; --k; }             \
                q[k] = val;                                                                 \
            }                                                                               \
        }                                                                                   \
    }                                                                                       \
    static void NAME(const R* v, int64_t M, R* v1, R* v2, int64_t* j1) {                    \
        if (2 * 64 <= M) {                                                                  \
            R best = v[0], second; int64_t p1 = 0, p2 = -1, j;                              \
            second = -INFINITY;                                                             \
            for (j = 1; j < M; ++j) {                                                       \
                if (v[j] > best) { second = best; best = v[j]; p1 = j; p2 = -1; }           \
                else if (v[j] == best) { if (p2 < 0) p2 = j; second = best; }               \
                else if (v[j] > second) second = v[j];                                      \
            }                                                                               \
            *v1 = best; *v2 = second;                                                       \
            *j1 = (p2 >= 0 && !(p1 == 0 && p2 == 1)) ? p2 : p1;                             \
        } else {                                                                            \
            NAME##_pair q[128];                                                             \
            int lg = 0; while (((int64_t)1 << (lg + 1)) <= M) lg++;                         \
            for (int64_t j = 0; j < M; ++j) { q[j].v = v[j]; q[j].i = j; }                  \
            NAME##_introselect(q, 0, 1, M, 2 * lg);                                         \
            *v1 = q[0].v; *v2 = q[1].v; *j1 = q[0].i;                                       \
        }                                                                                   \
    }

DEFINE_TOPK(float, topk_row_f)
DEFINE_TOPK(double, topk_row_d)

/*
 * One problem.  cost points at the batch base; off0 = b*stride_b.
 * stats: [bidding rounds, row-bids, tied row-bids, unassigned at exit]
 */
#define DEFINE_SOLVER(R, NAME, LOADER, TOPK)                                                      \
    static void NAME(const void* cost, int dtype, int64_t off0, int64_t stride_n,           \
                     int64_t N, int64_t M, const double* eps, int n_eps, int max_iter,      \
                     int tie_rule, int64_t* assign, R* P, int64_t* stats, int inner_threads) { \
        int64_t* owner = (int64_t*)malloc(sizeof(int64_t) * (size_t)(M > 0 ? M : 1));       \
        int64_t* active = (int64_t*)malloc(sizeof(int64_t) * (size_t)(N > 0 ? N : 1));      \
        int64_t* bidcol = (int64_t*)malloc(sizeof(int64_t) * (size_t)(N > 0 ? N : 1));      \
        R* bid = (R*)malloc(sizeof(R) * (size_t)(N > 0 ? N : 1));                           \
        int64_t* winner = (int64_t*)malloc(sizeof(int64_t) * (size_t)(M > 0 ? M : 1));      \
        int64_t* tied = (int64_t*)calloc((size_t)(N > 0 ? N : 1), sizeof(int64_t));         \
        int64_t rounds = 0, rowbids = 0, ties = 0, i, j, k;                                 \
        for (j = 0; j < M; ++j) { P[j] = (R)0; winner[j] = -1; }                            \
        for (i = 0; i < N; ++i) assign[i] = -1;                                             \
        for (int ph = 0; ph < n_eps; ++ph) {                                                \
            const R e = (R)eps[ph];                                                         \
            const R win_tol = (R)1e-5;                                                      \
            for (i = 0; i < N; ++i) assign[i] = -1;                                         \
            for (j = 0; j < M; ++j) owner[j] = -1;                                          \
            for (int it = 0; it < max_iter; ++it) {                                         \
                int64_t K = 0;                                                              \
                for (i = 0; i < N; ++i) if (assign[i] == -1) active[K++] = i;               \
                if (K == 0) break;                                                          \
                rounds++; rowbids += K;                                                     \
                /* bids: independent per row, read the round-start prices */               \
                _Pragma("omp parallel for schedule(static) num_threads(inner_threads) if(inner_threads > 1 && K >= 64)") \
                for (k = 0; k < K; ++k) {                                                   \
                    R* buf = (R*)malloc(sizeof(R) * (size_t)M);                             \
                    LOADER(cost, dtype, off0 + active[k] * stride_n, M, buf);               \
                    R v1, v2; int64_t j1, jj;                                               \
                    for (jj = 0; jj < M; ++jj) buf[jj] = buf[jj] - P[jj];                   \
                    TOPK(buf, M, &v1, &v2, &j1);                                            \
                    tied[k] = (v2 == v1) ? 1 : 0;                                  \
                    R inc = (v1 - v2) + e;                                                  \
                    bidcol[k] = j1;                                                         \
                    bid[k] = P[j1] + inc;                                                   \
                    free(buf);                                                              \
                }                                                                           \
                for (k = 0; k < K; ++k) ties += tied[k];                                    \
                /* scatter_reduce amax, include_self */                                     \
                for (k = 0; k < K; ++k) { j = bidcol[k]; if (bid[k] > P[j]) P[j] = bid[k]; } \
                /* election: ascending rows, last writer wins (tie_rule 0, the           \
                   reference); tie_rule 1 keeps the first, i.e. the lowest row */           \
                for (k = 0; k < K; ++k) {                                                   \
                    j = bidcol[k];                                                          \
                    R d = bid[k] - P[j]; if (d < 0) d = -d;                                 \
                    if (d < win_tol && (tie_rule == 0 || winner[j] < 0)) winner[j] = active[k]; \
                }                                                                           \
                /* ownership transfer; every won column appears once */                     \
                for (k = 0; k < K; ++k) {                                                   \
                    j = bidcol[k];                                                          \
                    int64_t w = winner[j];                                                  \
                    if (w < 0) continue;                                                    \
                    winner[j] = -1;                                                         \
                    int64_t prev = owner[j];                                                \
                    if (prev != -1) assign[prev] = -1;                                      \
                    owner[j] = w;                                                           \
                    assign[w] = j;                                                          \
                }                                                                           \
            }                                                                               \
        }                                                                                   \
        int64_t un = 0; for (i = 0; i < N; ++i) un += (assign[i] == -1);                    \
        stats[0] = rounds; stats[1] = rowbids; stats[2] = ties; stats[3] = un;              \
        free(owner); free(active); free(bidcol); free(bid); free(winner); free(tied);      \
    }

DEFINE_SOLVER(float, solve_one_f, load_row_f, topk_row_f)
DEFINE_SOLVER(double, solve_one_d, load_row_d, topk_row_d)

/*
 * Batch entry point.  cost: (B,N,M) with element strides (stride_b, stride_n, 1).
 * assign_out: B*N int64 (-1 = unassigned).  prices_out: B*M float (fp32/fp16/
 * bf16 input) or double (fp64 input).  stats_out: B*4 int64.
 * Returns 0 on success, 1 on a bad argument.
 */
int ela_oracle_solve(const void* cost, int dtype, int64_t B, int64_t N, int64_t M,
                     int64_t stride_b, int64_t stride_n, const double* eps, int n_eps,
                     int max_iter, int tie_rule, int64_t* assign_out, void* prices_out,
                     int64_t* stats_out, int nthreads) {
    if (B < 0 || N < 0 || M < 0 || n_eps < 1 || max_iter < 0) return 1;
    if (dtype < 0 || dtype > 3) return 1;
    if (tie_rule != 0 && tie_rule != 1) return 1;
    if (N > 0 && M < 2) return 1; /* torch.topk(k=2) needs two columns */
    if (nthreads < 1) nthreads = 1;
    int outer = (B >= nthreads) ? nthreads : 1;
    int inner = (outer == 1) ? nthreads : 1;
    int64_t b;
#pragma omp parallel for schedule(dynamic, 1) num_threads(outer) if (outer > 1)
    for (b = 0; b < B; ++b) {
        if (dtype == ELA_F64)
            solve_one_d(cost, dtype, b * stride_b, stride_n, N, M, eps, n_eps, max_iter,
                        tie_rule, assign_out + b * N, (double*)prices_out + b * M, stats_out + 4 * b, inner);
        else
            solve_one_f(cost, dtype, b * stride_b, stride_n, N, M, eps, n_eps, max_iter,
                        tie_rule, assign_out + b * N, (float*)prices_out + b * M, stats_out + 4 * b, inner);
    }
    return 0;
}

/*
 * One round's bids (the checker of ela_auction_compute_bids): for every row
 * whose assignment is -1 (or every row when assign is NULL), the column
 * torch.topk(k=2) picks on v = (-c) - P and the increment (v1 - v2) + eps,
 * exactly as one round of AuctionTorch.solve computes them
 * (torch_backend.py:65-88); other rows get column -1 and increment 0, as the
 * reference's compute_bids kernel writes (src/csrc/kernels.cu:53-57).
 * prices: B*M float (double for fp64) or NULL (zeros).  inc_out: B*N float
 * (double for fp64).  Returns 0, or 1 on a bad argument.
 */
#define DEFINE_BIDS(R, NAME, LOADER, TOPK)                                                       \
    static void NAME(const void* cost, int dtype, int64_t off0, int64_t stride_n, int64_t N,    \
                     int64_t M, const R* P, const int64_t* assign, double eps, int64_t* idx,    \
                     R* inc) {                                                                   \
        R* buf = (R*)malloc(sizeof(R) * (size_t)M);                                             \
        for (int64_t i = 0; i < N; ++i) {                                                       \
            if (assign && assign[i] != -1) { idx[i] = -1; inc[i] = (R)0; continue; }            \
            LOADER(cost, dtype, off0 + i * stride_n, M, buf);                                   \
            for (int64_t j = 0; j < M; ++j) buf[j] = buf[j] - (P ? P[j] : (R)0);                \
            R v1, v2; int64_t j1;                                                               \
            TOPK(buf, M, &v1, &v2, &j1);                                                        \
            idx[i] = j1;                                                                        \
            inc[i] = (v1 - v2) + (R)eps;                                                        \
        }                                                                                       \
        free(buf);                                                                              \
    }

DEFINE_BIDS(float, bids_one_f, load_row_f, topk_row_f)
DEFINE_BIDS(double, bids_one_d, load_row_d, topk_row_d)

int ela_oracle_bids(const void* cost, int dtype, int64_t B, int64_t N, int64_t M, int64_t stride_b,
                    int64_t stride_n, const void* prices, const int64_t* assign, double eps,
                    int64_t* idx_out, void* inc_out) {
    if (B < 0 || N < 0 || M < 0 || dtype < 0 || dtype > 3) return 1;
    if (N > 0 && M < 2) return 1;
    for (int64_t b = 0; b < B; ++b) {
        const int64_t* a = assign ? assign + b * N : NULL;
        if (dtype == ELA_F64)
            bids_one_d(cost, dtype, b * stride_b, stride_n, N, M, prices ? (const double*)prices + b * M : NULL, a,
                       eps, idx_out + b * N, (double*)inc_out + b * N);
        else
            bids_one_f(cost, dtype, b * stride_b, stride_n, N, M, prices ? (const float*)prices + b * M : NULL, a,
                       eps, idx_out + b * N, (float*)inc_out + b * N);
    }
    return 0;
}
