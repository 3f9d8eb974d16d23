/*
 * ela_auction.h -- C ABI of the B200 auction linear-assignment solver
 * (libela_auction.so, built from efficient-linear-assignment_b200/csrc/ela_auction.cu).
 *
 * Plain pointers and sizes only; no torch types.  All pointers passed to the
 * solve call are DEVICE pointers on the current CUDA device except the epsilon
 * schedule, which is a host array.  Work is enqueued on `stream` and the call
 * returns without waiting for it.
 *
 * Reference interfaces this ABI replaces (paths inside the reference project):
 *   - pybind11 solve_auction_cuda(cost, epsilon, max_iter, persistent_mode)
 *       src/csrc/interface.cpp:4,64 ; src/csrc/kernels.cu:449-585
 *     -> ela_auction_solve (the whole solve, every round on the device)
 *   - the backend plug-in AuctionCPPCCUDA.solve(cost) -> (assignment, prices)
 *       src/efficient_linear_assignment/auction/cpp_backend.py:24-40
 *     -> reached from Python through the ctypes binding in the package's _lib.py
 *   - the device scratch the reference allocates inside solve_auction_cuda
 *       src/csrc/kernels.cu:461-472
 *     -> caller-owned workspace sized by ela_auction_workspace_bytes
 */
#ifndef ELA_AUCTION_H
#define ELA_AUCTION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by the calls below and written to *status_out. */
enum {
    ELA_OK = 0,
    ELA_ERR_ARGUMENT = 1,    /* bad size, stride, dtype, schedule or pointer    */
    ELA_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed             */
    ELA_ERR_TIMEOUT = 3,     /* a device-side wait ran past its limit            */
    ELA_ERR_UNSUPPORTED = 4, /* valid arguments this build cannot run (size)     */
    ELA_ERR_INTERNAL = 5     /* a device-side consistency check failed           */
};

/* Element type of the cost matrix. */
enum { ELA_DTYPE_F32 = 0, ELA_DTYPE_F16 = 1, ELA_DTYPE_BF16 = 2, ELA_DTYPE_F64 = 3 };

/* Kernel choice.  AUTO picks by batch and problem size.
 *   CTA      one CTA per problem (batches of small problems)
 *   GRID     several co-resident CTAs per problem, bids exchanged through global memory
 *   CLUSTER  one thread-block cluster per problem, bids exchanged through
 *            distributed shared memory (few large problems; needs M >= 128) */
enum { ELA_PATH_AUTO = 0, ELA_PATH_CTA = 1, ELA_PATH_GRID = 2, ELA_PATH_CLUSTER = 3 };

/* Row tie rule of the election.  Among the bids on one column that lie within
 * 1e-5 of its new price, ELA_TIE_HIGHEST_ROW (the reference's rule: torch's
 * index_put_ with ascending rows keeps the last writer,
 * src/efficient_linear_assignment/auction/torch_backend.py:126-136) elects the
 * highest row; ELA_TIE_LOWEST_ROW elects the lowest.  Only HIGHEST_ROW gives
 * the reference's indices; LOWEST_ROW is an equally valid auction (same bids,
 * same prices, same epsilon-optimality bound). */
enum { ELA_TIE_HIGHEST_ROW = 0, ELA_TIE_LOWEST_ROW = 1 };

/* Library ABI version (major*100 + minor). */
int ela_auction_version(void);

/* Human-readable name of a status code. */
const char* ela_status_string(int status);

/*
 * Bytes of device workspace ela_auction_solve needs for these sizes and path
 * (on the current device).  Returns 0 if the arguments are invalid.
 */
size_t ela_auction_workspace_bytes(int dtype, int64_t B, int64_t N, int64_t M, int path);

/*
 * Solve B independent N x M assignment problems (minimise total cost) with the
 * Jacobi auction of the reference torch backend
 * (src/efficient_linear_assignment/auction/torch_backend.py:9-159).
 *
 *   cost        device, element (b,i,j) at cost[b*stride_b + i*stride_n + j]
 *   dtype       ELA_DTYPE_*; fp16/bf16 are widened to fp32, prices and bids are
 *               fp32 (fp64 for ELA_DTYPE_F64)
 *   eps_schedule, n_eps
 *               host array of n_eps >= 1 epsilons, each > 0.  n_eps == 1 is the
 *               reference's constant-epsilon solve; n_eps > 1 runs one full
 *               solve per epsilon, each starting from the previous prices
 *   max_iter    bidding rounds allowed per epsilon (reference default 1000)
 *   path        ELA_PATH_* (launch shape; every path gives the same results)
 *   tie_rule    ELA_TIE_* (ELA_TIE_HIGHEST_ROW reproduces the reference)
 *   assign_out  device int64[B*N]; column of each row, -1 if unassigned
 *   prices_out  device float[B*M] (double[B*M] for ELA_DTYPE_F64)
 *   stats_out   device int64[B*4] or NULL: per problem
 *               {bidding rounds, row-bids, 0, unassigned rows at exit}
 *   status_out  device int32[1] or NULL; receives ELA_OK or a device-side error
 *   workspace   device, >= ela_auction_workspace_bytes(...) bytes, 256-byte aligned
 *   stream      cudaStream_t (NULL = legacy default stream)
 *
 * Requires M >= 2 when N > 0 (top-2 bidding), stride_n >= M, stride_b >= N*stride_n.
 * Returns ELA_OK once the work is enqueued, or an error code.
 */
int ela_auction_solve(const void* cost, int dtype, int64_t B, int64_t N, int64_t M,
                      int64_t stride_b, int64_t stride_n, const double* eps_schedule,
                      int n_eps, int max_iter, int path, int tie_rule, int64_t* assign_out,
                      void* prices_out, int64_t* stats_out, int32_t* status_out,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * The solve of the reference's padded problem without building it.  The
 * reference requires N and M to be multiples of 8 and pads other shapes with
 * pad_input (src/efficient_linear_assignment/utils.py:32-105): real rows get
 * cost 1e9 on the added columns, added rows get 1e9 on the real columns and 0
 * on the added columns (1e9 when only rows are added), 1e9 rounded to the
 * cost's dtype (fp16: +inf; the reference's pad_input refuses fp16 because
 * torch.full cannot store 1e9 there).  This call solves that (B, N', M') problem, N' and M' the
 * next multiples of `multiple`, from the unpadded (B, N, M) cost: the padding
 * entries are synthesised by the kernel's loaders and never stored.
 *
 * Arguments as ela_auction_solve, with N, M, strides describing the unpadded
 * cost; assign_out holds B*N' entries (row-major (B, N'); the caller keeps the
 * first N of each problem, as unpad_result does), prices_out B*M'.  Size the
 * workspace with ela_auction_workspace_bytes(dtype, B, N', M', path).  Padded
 * shapes use the one-CTA or grid kernel (scalar loads); ELA_PATH_CLUSTER
 * returns ELA_ERR_UNSUPPORTED.  Shapes that need no padding run
 * ela_auction_solve unchanged.
 */
int ela_auction_solve_padded(const void* cost, int dtype, int64_t B, int64_t N, int64_t M,
                             int64_t stride_b, int64_t stride_n, int multiple, const double* eps_schedule,
                             int n_eps, int max_iter, int path, int tie_rule, int64_t* assign_out,
                             void* prices_out, int64_t* stats_out, int32_t* status_out,
                             void* workspace, size_t workspace_bytes, void* stream);

/*
 * The IMLE backward's second solve without its dense input.  The reference's
 * AuctionIMLE.backward solves the target cost `cost_matrix + lambda *
 * grad_output` (src/efficient_linear_assignment/auction/api.py:106-111), a
 * (B,N,M) tensor it builds first.  This call solves the same problem from the
 * two tensors: every cost the kernel reads is cost + lam * grad, rounded as
 * torch evaluates it in the input dtype (lam * grad rounded to the dtype,
 * then the sum rounded), so results equal ela_auction_solve on the
 * materialised sum.  grad has cost's dtype, shape and strides (B*stride_b
 * layout); both device pointers.  Other arguments as ela_auction_solve.  It
 * runs on the one-CTA and grid kernels; ELA_PATH_CLUSTER, or a size only the
 * cluster kernel fits, returns ELA_ERR_UNSUPPORTED (the caller then solves the
 * materialised sum).
 */
int ela_auction_solve_sum(const void* cost, const void* grad, double lam, int dtype, int64_t B, int64_t N,
                          int64_t M, int64_t stride_b, int64_t stride_n, const double* eps_schedule, int n_eps,
                          int max_iter, int path, int tie_rule, int64_t* assign_out, void* prices_out,
                          int64_t* stats_out, int32_t* status_out, void* workspace, size_t workspace_bytes,
                          void* stream);

/*
 * Auction on implicit low-rank costs C = Q K^T, the reference's planned
 * solve_implicit(Q, K, ...) (optimization_plan.md:11-22): cost tiles are
 * computed on the tensor cores (tcgen05.mma, fp32 accumulation) in every
 * round from Q (B, N, D) and K (B, M, D), never stored.  Q and K: device,
 * contiguous, bf16 or fp16 (dtype), 16-byte aligned; D a multiple of 16 in
 * [16, 256]; 128 <= M <= 512.  One CTA per problem.  Minimises sum C[i][a(i)]
 * with the reference's round (eps_schedule, max_iter, tie_rule as in
 * ela_auction_solve).  assign_out int64[B*N] (-1 = unassigned), prices_out
 * float[B*M], stats_out int64[B*4] or NULL, status_out int32[1] (required).
 * Each cost value is the fp32 result of one fixed MMA instruction sequence,
 * so the solve equals ela_auction_solve on the matrix that
 * ela_auction_implicit_costs writes; that matrix is Q K^T up to fp32
 * rounding of the dot products.
 */
int ela_auction_solve_implicit(const void* Q, const void* K, int dtype, int64_t B, int64_t N, int64_t M, int64_t D,
                               const double* eps_schedule, int n_eps, int max_iter, int tie_rule,
                               int64_t* assign_out, float* prices_out, int64_t* stats_out, int32_t* status_out,
                               void* stream);

/*
 * The costs ela_auction_solve_implicit uses, written out: cost_out float
 * [B*N*M] receives C = Q K^T computed by the same tensor-core instructions.
 * Test and inspection aid for the implicit solve (same size limits).
 */
int ela_auction_implicit_costs(const void* Q, const void* K, int dtype, int64_t B, int64_t N, int64_t M, int64_t D,
                               float* cost_out, int32_t* status_out, void* stream);

/*
 * One round's bids, the reference's compute_bids(benefits, prices,
 * assignment, best_idx, increments, epsilon) (src/csrc/interface.cpp:31-40,
 * launch_bid_kernel_cuda in src/csrc/kernels.cu:420-445): for every row of
 * every problem whose assignment is -1, the column it bids on and its
 * increment (v1 - v2) + epsilon, where v = -cost - price over the row and
 * (v1, v2) are its two largest values; the column is the one the torch
 * backend's topk picks (torch_backend.py:65-88), ties included.  Rows already
 * assigned get column -1 and increment 0.  cost as in ela_auction_solve;
 * prices: device, contiguous B x M, float (double for fp64 costs), or NULL
 * for all zeros; assignment: device int64 B x N, or NULL (every row bids);
 * best_idx_out int64 B x N, increments_out float (double for fp64) B x N.
 * One streaming pass over the rows (HBM-bound).  The problem's prices are
 * staged in shared memory, so M is limited to what fits (ELA_ERR_UNSUPPORTED
 * beyond).  Work is enqueued on `stream`; returns a status (ELA_OK ...).
 */
int ela_auction_compute_bids(const void* cost, int dtype, int64_t B, int64_t N, int64_t M, int64_t stride_b,
                             int64_t stride_n, const void* prices, const int64_t* assignment, double epsilon,
                             int64_t* best_idx_out, void* increments_out, void* stream);

/*
 * Limit, in nanoseconds, on every device-side wait of the grid path (each
 * round's exchange of bids between the CTAs that share one problem).  A wait that
 * runs out writes ELA_ERR_TIMEOUT to *status_out and the kernel returns.
 * Default 2 s.  Process-wide setting.
 */
void ela_auction_set_wait_limit_ns(uint64_t ns);

/*
 * Test hook for the timeout path.  When `on` is nonzero, CTA 0 of every group
 * of the grid path, and of every team of clusters of the cluster path, never
 * publishes its first exchanged round's bids, so every CTA's bounded wait for
 * them runs out and the solve ends with ELA_ERR_TIMEOUT
 * (no fault, no hang; the CUDA context stays usable).  Process-wide setting.
 */
void ela_auction_debug_skip_arrive(int on);

/*
 * Size of the fixed device scratch array behind ela_auction_solve_noalloc:
 * 4 MiB, held in every GPU's memory from library load until process exit.
 */
#define ELA_NOALLOC_SCRATCH_BYTES (4u << 20)

/*
 * ela_auction_solve without a workspace argument, for callers that cannot
 * allocate device memory themselves: hosts that own the GPU through a
 * pre-reserved memory pool in which a cudaMalloc would fail or fragment, code
 * that must not trigger cudaMalloc's implicit device synchronisation, and
 * foreign-language bindings with no access to a device allocator.  It has no
 * counterpart in the reference, which allocates its scratch inside the call.
 *
 * Arguments, results and status codes are those of ela_auction_solve; the
 * caller still provides cost, assignment, price, stats and status buffers.
 * The solve's scratch lives in a library-owned static device array of
 * ELA_NOALLOC_SCRATCH_BYTES bytes; sizes whose scratch would not fit return
 * ELA_ERR_UNSUPPORTED before any work is enqueued.  The call allocates
 * nothing (no cudaMalloc, no cudaFree, no allocating library routine).
 *
 * The first call on a device (and the first after the device's context is
 * replaced, e.g. by cudaDeviceReset) looks up that context's address of the
 * array (cudaGetSymbolAddress, with the device current); make that first call
 * before any stream capture.  All calls on a device share the one array and
 * each call clears the part it uses, so calls whose work overlaps on the GPU
 * (different streams, or concurrent host threads) race and give wrong
 * results: order them, e.g. on one stream.
 */
int ela_auction_solve_noalloc(const void* cost, int dtype, int64_t B, int64_t N, int64_t M,
                              int64_t stride_b, int64_t stride_n, const double* eps_schedule,
                              int n_eps, int max_iter, int path, int tie_rule,
                              int64_t* assign_out, void* prices_out, int64_t* stats_out,
                              int32_t* status_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ELA_AUCTION_H */
