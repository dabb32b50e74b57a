/*
 * sandmuon_b200.h -- C-ABI of libsandmuon_b200.so, the B200 (sm_100a) engine
 * behind the drop-in `sandmuon_b200` optimizer package.
 *
 * Conventions
 *   - Every entry point is `extern "C"`, takes plain pointers / sizes / POD
 *     structs, and returns an int status: 0 = success, otherwise one of the
 *     SM_ERR_* codes below.  `sm_last_error()` returns a thread-local message
 *     describing the last failure on the calling thread.
 *   - Every device operation is stream-ordered on the caller-supplied
 *     `stream` (a cudaStream_t passed as void*; NULL = legacy default stream).
 *   - The library never allocates device memory.  The caller (PyTorch in the
 *     Python package) allocates every tensor and workspace and passes them in.
 *     The library keeps no references to caller memory after a call returns,
 *     except inside an `SmPlan`, which records the pointers given at creation
 *     and must be destroyed (or rebuilt) when any of them is freed.
 *   - Entry points are reentrant; a plan must not be stepped concurrently from
 *     two threads.
 *
 * Reference interfaces replaced (paths within the SandMuon project):
 *   sm_stats_accumulate  <- forward hook `a_sum += x^2.sum(0)`, `a_first_sum += x.sum(0)`
 *                           (sandmuon/optimizer.py:151-168) and the cotangent hook
 *                           `b_sum += delta^2.sum(0)` (sandmuon/optimizer.py:170-179)
 *   sm_plan_*            <- DiagonalWeightedPE.step matrix path
 *                           (sandmuon/optimizer.py:224-266, 283-316) including
 *                           _finish_a / _finish_b (:182-222), rank1_whiten (:38-45),
 *                           _s8_fp32 (:69-93), rank1_mapback (:48-60),
 *                           _graft_direction (:63-66)
 *   sm_s8_polar          <- _s8_fp32 (sandmuon/optimizer.py:69-93) on a batch
 *   sm_adamw_multi       <- auxiliary AdamW loop (sandmuon/optimizer.py:268-281)
 *   sm_gemm_bf16         <- the dense products inside _s8_fp32 (x @ x.mT, gram @ gram,
 *                           p @ x; sandmuon/optimizer.py:79-91); exported for unit tests
 */
#ifndef SANDMUON_B200_H
#define SANDMUON_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SM_ABI_VERSION 3

/* status codes */
#define SM_OK 0
#define SM_ERR_ARG 1          /* invalid argument (shape, dtype, alignment, null) */
#define SM_ERR_CUDA 2         /* a CUDA runtime call failed */
#define SM_ERR_WORKSPACE 3    /* workspace too small */
#define SM_ERR_UNSUPPORTED 4  /* device is not sm_100 or feature unavailable */
#define SM_ERR_DEVICE 5       /* a kernel reported a device-side error (timeout) */

/* element types accepted by sm_stats_accumulate */
#define SM_DTYPE_F32 0
#define SM_DTYPE_BF16 1
#define SM_DTYPE_F16 2
#define SM_DTYPE_F64 3

/* ---------------------------------------------------------------- basics */

/* ABI version (SM_ABI_VERSION). */
int sm_version(void);

/* Thread-local text of the last error reported on this thread ("" if none). */
const char* sm_last_error(void);

/* Checks the current device is a B200-class sm_100 GPU and warms the library's
 * kernels (sets their shared-memory attributes).  Returns SM_ERR_UNSUPPORTED
 * on other devices. */
int sm_init_device(void);

/* Reads and clears the device-side status word that bounded waits inside the
 * library's kernels set on timeout (0 = no error).  Synchronises `stream`. */
int sm_device_status(int* status_out, void* stream);

/* --------------------------------------------------- N1: hook statistics */

/* Bytes of workspace sm_stats_accumulate needs for an [n_rows, n_cols] input. */
size_t sm_stats_workspace_bytes(int64_t n_rows, int64_t n_cols);

/* Column statistics of a 2-D row block, accumulated in place:
 *   sum_sq[c] += sum_r float(x[r, c])^2
 *   sum[c]    += sum_r float(x[r, c])        (skipped when sum == NULL)
 * x[r, c] lives at rows + (r * row_stride + c * col_stride) * elem_size.
 * Deterministic: a fixed two-pass reduction order, no float atomics.
 * Replaces the forward hook (sandmuon/optimizer.py:156-168) and the cotangent
 * hook (sandmuon/optimizer.py:170-179). */
int sm_stats_accumulate(const void* rows, int dtype, int64_t n_rows, int64_t n_cols,
                        int64_t row_stride, int64_t col_stride, float* sum_sq, float* sum,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Same statistics as sm_stats_accumulate, for callers that cannot allocate
 * device memory.  No counterpart in the reference: its hooks always let torch
 * allocate temporaries.  Some callers hold only the tensors they were handed:
 * a statistics hook running inside another framework's training step, where
 * that framework's allocator owns the rest of HBM (a caching allocator usually
 * reserves most of it), so a raw cudaMalloc can fail or fragment its pool, and
 * cudaFree synchronises the whole device in the middle of the step.
 * The partial sums go to one library-owned scratch array of
 * SM_STATS_NOALLOC_SCRATCH_FLOATS floats (2 MiB) that every GPU which loads
 * the library keeps until the process exits.  Limit: n_cols <=
 * SM_STATS_NOALLOC_MAX_COLS; larger inputs return SM_ERR_ARG before any device
 * work.  The first call on a device looks the array's device address up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * Each device has its own copy of the array, shared by every call on that
 * device and keeping what the last call left there.  A call overwrites the
 * partial sums before reading them and clears the completion counters it
 * uses (cudaMemsetAsync on its stream, which allocates nothing), so nothing
 * from an earlier call leaks into a later one; but calls that overlap on the
 * GPU (for example on two streams) race on the array and may return wrong
 * sums: keep them in one stream order. */
#define SM_STATS_NOALLOC_SCRATCH_FLOATS (1 << 19)
#define SM_STATS_NOALLOC_MAX_COLS (SM_STATS_NOALLOC_SCRATCH_FLOATS / 2)
int sm_stats_accumulate_noalloc(const void* rows, int dtype, int64_t n_rows, int64_t n_cols,
                                int64_t row_stride, int64_t col_stride, float* sum_sq, float* sum,
                                void* stream);

/* ------------------------------------------------------ optimizer plan */

/* One selected weight matrix (a torch Linear weight, shape [d_out, d_in],
 * FP32, row-major and contiguous) and its persistent state. */
typedef struct {
    float* weight;        /* [d_out, d_in] updated in place                  */
    float* momentum;      /* [d_out, d_in] FP32 momentum_buffer              */
    float* export_to;     /* NULL, or [d_out, d_in]: the updated weight (or its
                             BF16 delta, SM_EXPORT_BF16_DELTA) is also
                             written here (a rank's all-gather send slot)    */
    int32_t d_out;
    int32_t d_in;
    int32_t a_stat;       /* index into the A-statistic table (shared q/k/v)  */
    int32_t b_stat;       /* index into the B-statistic table                 */
} SmMatrixSpec;

/* One activation (A) or cotangent (B) statistic vector and its EMA state. */
typedef struct {
    float* sum;           /* a_sum / b_sum  [n] (zeroed by the step)          */
    float* first_sum;     /* a_first_sum [n] (rank-one A only, else NULL)     */
    float* ema;           /* a_ema / b_ema [n]                                */
    float* mean_ema;      /* a_mean_ema [n] (rank-one A only, else NULL)      */
    int32_t n;            /* vector length                                    */
    int32_t kind;         /* SM_STAT_A_DIAG, SM_STAT_A_RANK1 or SM_STAT_B     */
} SmStatSpec;

#define SM_STAT_A_DIAG 0
#define SM_STAT_A_RANK1 1
#define SM_STAT_B 2

/* What the step writes to SmMatrixSpec.export_to (when not NULL). */
#define SM_EXPORT_WEIGHTS 0     /* float [d_out, d_in]: the updated weight                   */
#define SM_EXPORT_BF16_DELTA 1  /* bf16 [d_out, d_in]: D = bf16(lr * direction); the weight is
                                   updated as W -= float(D), exactly what
                                   sm_apply_bf16_delta_multi does on other ranks            */

typedef struct {
    const SmMatrixSpec* matrices;
    int32_t n_matrices;
    const SmStatSpec* stats;
    int32_t n_stats;
    float statistic_beta;    /* 0.97 (sandmuon/optimizer.py:123)            */
    float momentum;          /* 0.8  (sandmuon/optimizer.py:139)            */
    int32_t export_mode;     /* SM_EXPORT_WEIGHTS or SM_EXPORT_BF16_DELTA    */
} SmPlanSpec;

typedef struct SmPlan SmPlan;

/* Per-step dynamic inputs. Arrays are host memory, indexed like the spec. */
typedef struct {
    const float* const* grads;   /* [n_matrices] device pointers to FP32 grads, same
                                    layout as the weight                           */
    const float* lrs;            /* [n_matrices] learning rate of each matrix      */
    const int64_t* counts;       /* [n_stats] rows accumulated into each statistic */
    const int32_t* ema_init;     /* [n_stats] 1 = first step: EMA <- value (copy)  */
    const int64_t* device_counts; /* NULL, or a DEVICE array [n_stats] of row counts
                                     that replaces `counts` in the arithmetic (the
                                     all-reduced counts of a data-parallel group,
                                     read without a host synchronisation)         */
} SmStepArgs;

/* Workspace bytes a plan needs (256-byte aligned pointer required). */
int sm_plan_workspace_bytes(const SmPlanSpec* spec, size_t* bytes_out);

/* Builds a plan: groups matrices by oriented S8 shape (rows <= cols), lays the
 * workspace out, zeroes its padding on `stream`, and encodes TMA descriptors. */
int sm_plan_create(const SmPlanSpec* spec, void* workspace, size_t workspace_bytes,
                   void* stream, SmPlan** plan_out);

/* One optimizer step for every matrix of the plan:
 *   finish statistics (EMA, inverse square roots, rank-one factors; sums zeroed)
 *   -> Nesterov momentum -> two-sided whitening -> 5-stage S8 polynomial
 *   (stages 1-4 compensated BF16 -- hi/lo operand planes, three products --
 *   and stage 5 plain BF16, FP32 accumulation throughout, on tcgen05)
 *   -> mapback -> Frobenius graft to sqrt(d_out) -> W -= lr * direction. */
int sm_plan_step(SmPlan* plan, const SmStepArgs* args, void* stream);

/* Graph replay (default on): from a plan's second step on, sm_plan_step
 * launches its kernels as one CUDA graph, captured once on a private stream
 * and re-captured only when the gradients' 16-byte alignment pattern changes;
 * the per-step arguments travel in a descriptor table uploaded from host
 * memory before each replay.  Results are identical either way.  A step
 * issued on a stream that is itself being captured returns
 * SM_ERR_UNSUPPORTED.  enabled = 0 launches every kernel individually. */
int sm_plan_set_replay(SmPlan* plan, int enabled);

/* Weight exchange by the update kernel itself (a sharded step; no
 * counterpart in the single-device reference, which has no exchange).  Each
 * rank keeps the selected matrices in one flat buffer of the same layout;
 * from the next step on, every weight the plan updates inside
 * [local_base, local_base + bytes) is also stored at the same offset from
 * each of the n_peers peer_bases: the other ranks' copies of that buffer,
 * mapped into this device's address space with sm_ipc_open.  The caller
 * orders the ranks' steps around it (a collective before the step, which
 * the statistic reduction is, and one after it, before any rank reads the
 * buffer).  n_peers = 0 turns it off.  At most 15 peers. */
int sm_plan_set_peers(SmPlan* plan, const void* local_base, int64_t bytes, const void* const* peer_bases,
                      int32_t n_peers);

/* CUDA IPC of a device buffer for sm_plan_set_peers.  sm_ipc_export writes
 * the 64-byte IPC handle of the allocation that holds ptr and ptr's byte
 * offset inside it; another process calls sm_ipc_open with the handle (on
 * its own current device: peer access over NVLink) and adds the offset to
 * the returned base; sm_ipc_close unmaps that base.  The exporter keeps the
 * allocation alive until every importer has closed it.  No multicast
 * mapping is made. */
int sm_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
int sm_ipc_open(const void* handle, void** base_out);
int sm_ipc_close(void* base);

/* Optional per-kernel-class timing with CUDA events (for the benchmark).
 * When enabled, sm_plan_step records an event pair around each launch;
 * sm_plan_timing_read synchronises, returns totals in ms per class and the
 * launch counts, and resets the accumulators.  Classes: see SM_TCLASS_*. */
#define SM_TCLASS_GEMM 0
#define SM_TCLASS_ELEMWISE 1
#define SM_TCLASS_STATS 2
#define SM_TCLASS_COUNT 3
int sm_plan_set_timing(SmPlan* plan, int enabled);
int sm_plan_timing_read(SmPlan* plan, double* ms_out, int64_t* launches_out,
                        double* gemm_flops_out);

/* Number of kernels one sm_plan_step launches. */
int sm_plan_launches_per_step(const SmPlan* plan, int64_t* out);

int sm_plan_destroy(SmPlan* plan);

/* ------------------------------------------------ multi-tensor copy */

typedef struct {
    void* dst;
    const void* src;
    int64_t bytes;        /* both pointers 16-byte aligned when bytes % 16 == 0 */
} SmCopySpec;

/* Copies every (src -> dst, bytes) of the list in one kernel launch (the
 * packing copies of a sharded step: gradients into the reduce-scatter's
 * buffer, momenta into the consolidation gather; no counterpart in the
 * single-device reference). */
int sm_copy_multi(const SmCopySpec* copies, int32_t count, void* stream);

/* One weight and the BF16 update delta to subtract from it. */
typedef struct {
    float* weight;
    const void* delta;    /* bf16, same element count as the weight */
    int64_t numel;
} SmDeltaSpec;

/* weight[i] -= float(delta[i]) for every (weight, delta) of the list, in one
 * kernel launch per 64 entries: how a rank applies the BF16 update deltas of
 * the matrices other ranks own (the sharded step's BF16 exchange; no
 * counterpart in the single-device reference). */
int sm_apply_bf16_delta_multi(const SmDeltaSpec* items, int32_t count, void* stream);

/* --------------------------------------------------------- S8 (batch) */

/* Workspace for sm_s8_polar on a batch of `batch` [rows, cols] matrices. */
size_t sm_s8_workspace_bytes(int32_t batch, int32_t rows, int32_t cols);

/* out[b] = S8(x[b]) for a contiguous FP32 batch [batch, rows, cols]; the same
 * oriented pipeline the plan runs (transposes when rows > cols), whose last
 * stage rounds its output to BF16. All-zero matrices give exact zeros.
 * Replaces _s8_fp32 (sandmuon/optimizer.py:69-93). */
int sm_s8_polar(const float* x, float* out, int32_t batch, int32_t rows, int32_t cols,
                void* workspace, size_t workspace_bytes, void* stream);

/* Tensor-core FLOPs sm_s8_polar executes on this device for such a batch:
 * the tiles actually computed (symmetric products: the upper block triangle
 * only) times three products in the compensated stages.  Host-side count. */
int sm_s8_executed_flops(int32_t batch, int32_t rows, int32_t cols, double* flops_out);

/* ------------------------------------------------- N8: auxiliary AdamW */

typedef struct {
    float* param;
    const float* grad;
    float* exp_avg;
    float* exp_avg_sq;
    int64_t numel;
    float bias_correction1;   /* 1 - beta1^step, computed on the host in double */
    float bias_correction2;   /* 1 - beta2^step                                  */
} SmAdamTensor;

/* One fused multi-tensor AdamW update (sandmuon/optimizer.py:268-281):
 *   m = b1 m + (1-b1) g ; v = b2 v + (1-b2) g^2
 *   u = (m / bc1) / (sqrt(v / bc2) + eps) ; p *= decay_factor ; p -= lr * u
 * decay_factor = 1 - lr * weight_decay (host-computed). */
int sm_adamw_multi(const SmAdamTensor* tensors, int32_t count, float lr, float beta1,
                   float beta2, float eps, float decay_factor, void* stream);

/* ------------------------------------------------- GEMM (unit testing) */

#define SM_EPI_F32 0        /* C = alpha * acc (FP32)                          */
#define SM_EPI_BF16 1       /* C = bf16(alpha * acc)                           */
#define SM_EPI_HILO 2       /* C_hi = bf16(alpha*acc), C_lo = bf16(rest)       */
#define SM_EPI_F32_NORM 3   /* FP32 store + per-tile sum of squares partials  */
#define SM_EPI_POLY 4       /* C = bf16(pa*I + pb*aux + pc*acc)                */
#define SM_EPI_POLY_HILO 5  /* P = pa*I + pb*(aux + aux_lo) + pc*acc -> hi/lo  */
#define SM_EPI_SYMMETRIC 0x100 /* flag: C is symmetric (M == N, K-major B); only the
                                 upper-triangular square tiles are computed and each
                                 off-diagonal tile also stores its transpose        */
#define SM_EPI_NORM_SLOTS 16   /* SM_EPI_F32_NORM partial sums per output tile   */

#define SM_GEMM_B_KMAJOR 1   /* layout flag: B is [batch, N, K] (C = A B^T), else [batch, K, N] */
#define SM_GEMM_A_MNMAJOR 2  /* layout flag: A is stored [batch, K, M] (A^T); needs an MN-major B */
#define SM_GEMM_PAIR 4       /* layout flag: CTA-pair tiles of 256 rows (tcgen05 cta_group::2);
                                needs M % 256 == 0 */
#define SM_GEMM_BN128 8      /* layout flag: 128-column tiles (a symmetric product on CTA
                                pairs then uses 256 x 128 block-row tiles) */

/* Batched C[b] = A[b] * op(B[b]) on tcgen05 tensor cores.
 *   A: [batch, M, K] BF16 row-major (K contiguous), or [batch, K, M] with
 *      SM_GEMM_A_MNMAJOR; a_lo != NULL selects the compensated 3-product mode
 *      (a_hi*b_lo + a_lo*b_hi + a_hi*b_hi), which then also needs b_lo.
 *   B: SM_GEMM_B_KMAJOR -> [batch, N, K] (C = A B^T); otherwise [batch, K, N].
 *   M % 128 == 0, N % 128 == 0, K % 64 == 0.
 *   out0/out1: outputs [batch, M, N] (out1 = lo plane for SM_EPI_HILO).
 *   alpha: device [batch] FP32 scales or NULL (1).  aux (and aux_lo for the
 *   hi/lo polynomial): BF16 [batch, M, N] for SM_EPI_POLY / SM_EPI_POLY_HILO.
 *   partials: device FP32 [batch, (M/TM)*(N/BN)*SM_EPI_NORM_SLOTS] for
 *   SM_EPI_F32_NORM, whose sum over a matrix is |C|_F^2.  Tile rows TM = 256
 *   with SM_GEMM_PAIR, else 128; tile columns BN = 128 with SM_GEMM_BN128,
 *   else TM for a symmetric output, else 256 when N % 256 == 0, else 128. */
int sm_gemm_bf16(const void* a_hi, const void* a_lo, const void* b_hi, const void* b_lo,
                 int layout, int32_t batch, int32_t m, int32_t n, int32_t k, int epilogue,
                 void* out0, void* out1, const float* alpha, const void* aux, const void* aux_lo,
                 float pa, float pb, float pc, float* partials, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SANDMUON_B200_H */
