/*
 * morpho_sm100.h -- C ABI of the B200 (sm_100a) MorphoAttention kernels.
 *
 * Plain C: no torch, no CUDA C++ types.  fp16 buffers are passed as void*, and the
 * CUDA stream as a void* holding a cudaStream_t (NULL = legacy default stream).
 * Every entry point is asynchronous on that stream and returns a status code; on
 * failure morpho_sm100_last_error() returns a message for the calling thread.
 *
 * Layouts (all row-major, contiguous, on the current CUDA device):
 *   X, out, grad_out, dX   fp16 [B, N, D]
 *   W_phi, dW_phi          fp16 [D, H*cube_m]   (used as X @ W_phi)
 *   W_V, dW_V              fp16 [D, D]          (used as X @ W_V)
 *   gate_q, gate_k, d_*    fp16 [H, cube_m]
 *   lse                    fp32 [B*H, N]        log2 domain: max_j s_ij + log2(sum_j 2^(s_ij - max))
 *
 * The two compute entry points replace the reference launchers
 *   attention_forward_kernel_launcher   (packages/morphottention/csrc/cuda/attention/attention.cuh:28-31,
 *                                         attention.cu:485-522)
 *   attention_backward_kernel_launcher  (attention.cuh:33-38, attention.cu:524-576)
 * with the same pointer arguments plus a caller-owned workspace.  Unlike the reference
 * launchers, cube_m and head_dim are run-time values and `causal` is honoured.
 */
#ifndef MORPHO_SM100_H
#define MORPHO_SM100_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MORPHO_API __attribute__((visibility("default")))
#else
#define MORPHO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MORPHO_OK 0
#define MORPHO_ERR_INVALID 1   /* bad shape, null pointer or unsupported (cube_m, head_dim) */
#define MORPHO_ERR_CUDA 2      /* a CUDA runtime or driver call failed */
#define MORPHO_ERR_WORKSPACE 3 /* workspace_bytes smaller than the *_workspace_size() answer */
#define MORPHO_ERR_DEVICE 4    /* current device is not sm_100 */
#define MORPHO_ERR_TIMEOUT 5   /* a kernel's bounded wait expired (see morpho_sm100_device_status) */
#define MORPHO_ERR_UNSUPPORTED 6 /* not available between these GPUs (e.g. no peer access) */

/* Hypercube projection phi = proj(z), z = X @ W_phi (reference morfology/cube.cuh:10-45, a
 * compile-time choice there, a run-time field here). */
#define MORPHO_PROJ_SIGMOID 0     /* 1 / (1 + e^-z)   (the reference default) */
#define MORPHO_PROJ_HARDTANH01 1  /* min(1, max(0, (z + 1) / 2)), gradient 1/2 on -1 < z < 1 */
#define MORPHO_PROJ_IDENTITY 2    /* z */

/* Score / aggregation (the reference's morfology/soft_morph.cuh:10-77, dead code there). */
#define MORPHO_SCORE_SOFTMAX 0   /* out = softmax_j(S_ij) . V (the reference attention kernels) */
#define MORPHO_SCORE_DILATION 1  /* out_ic = tau log sum_j exp((S_ij + V_jc) / tau): soft max-plus */
#define MORPHO_SCORE_EROSION 2   /* out_ic = -tau log sum_j exp(-(S_ij + V_jc) / tau): soft min-plus */

/* Gradient semantics of the backward. */
#define MORPHO_GRAD_FULL 0      /* true gradient of the forward (default) */
#define MORPHO_GRAD_REFERENCE 1 /* reference kernel semantics: query-code and query-bias
                                   terms are not propagated (attention.cu:447-451, :473-482) */

typedef struct morpho_problem {
    int32_t B;      /* batch */
    int32_t N;      /* tokens per sequence */
    int32_t D;      /* model dim, = H * head_dim */
    int32_t H;      /* heads */
    int32_t cube_m; /* hypercube width per head: 16, 32 or 64 */
    float scale;    /* softmax temperature */
    int32_t causal; /* 0 or 1 */
    int32_t grad_mode; /* MORPHO_GRAD_FULL or MORPHO_GRAD_REFERENCE (backward only) */
    int32_t projection; /* MORPHO_PROJ_* (0 = sigmoid) */
    int32_t mask_diag;  /* 1: also drop key j == query i (reference MORPHO_MASK_DIAG,
                           utils/declarations.cuh:79-82, attention.cu:131, :363); a query row
                           left with no key gives out = 0, lse = -FLT_MAX and no gradient */
    int32_t score;      /* MORPHO_SCORE_* (0 = softmax attention).  With DILATION / EROSION the
                           forward writes lse = 0 (not defined for them), grad_mode must be FULL,
                           and the backward returns dL/dtau as the last element of the fp32
                           weight-gradient bucket (see morpho_sm100_backward) */
    float tau;          /* temperature of DILATION / EROSION, > 0 (ignored for SOFTMAX) */
} morpho_problem_t;

/* Bytes of device workspace the forward / backward need for problem p (0 on invalid p). */
MORPHO_API size_t morpho_sm100_forward_workspace_size(const morpho_problem_t* p);
MORPHO_API size_t morpho_sm100_backward_workspace_size(const morpho_problem_t* p);

/* Forward: out = MorphoAttention(X), lse as above.
 * Replaces attention_forward_kernel_launcher (attention.cu:485-522). */
MORPHO_API int morpho_sm100_forward(const morpho_problem_t* p, const void* X, const void* W_phi, const void* gate_q,
                         const void* gate_k, const void* W_V, void* out, float* lse, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Backward of sum(out * grad_out): writes dX, dW_phi, d_gate_q, d_gate_k, dW_V (fp16).
 * The outputs are overwritten, not accumulated (no zero-fill needed, unlike
 * attention.cpp:93-98).  If dweights_f32 is non-NULL the weight gradients are written
 * there in fp32 instead -- layout [dW_phi (D*H*m) | dW_V (D*D) | d_gate_q (H*m) |
 * d_gate_k (H*m)], followed for the DILATION / EROSION scores by one element dL/dtau
 * (the temperature gradient of the reference's morfology/soft_morph.cuh:67-77, which exists
 * only in this fp32 form) -- and dW_phi/dW_V/d_gate_q/d_gate_k may be NULL; a data-parallel
 * caller all-reduces that bucket and then calls morpho_sm100_finalize_weight_grads.
 * Replaces attention_backward_kernel_launcher (attention.cu:524-576). */
MORPHO_API int morpho_sm100_backward(const morpho_problem_t* p, const void* grad_out, const void* X, const void* W_phi,
                          const void* gate_q, const void* gate_k, const void* W_V, const void* out,
                          const float* lse, void* dX, void* dW_phi, void* d_gate_q, void* d_gate_k, void* dW_V,
                          float* dweights_f32, void* workspace, size_t workspace_bytes, void* stream);

/* Training pair that keeps the projection between the two passes (no reference
 * counterpart: the reference recomputes it in the backward, attention.cu:524-576 calling
 * the same projection as the forward).  morpho_sm100_forward_save is morpho_sm100_forward
 * that leaves every projection output the backward needs -- codes, values, biases, phi and
 * the centered hi/lo key codes -- in the caller's `saved` buffer of
 * morpho_sm100_saved_bytes(p) bytes (no other workspace).  morpho_sm100_backward_saved is
 * morpho_sm100_backward that reads them from `saved` instead of running the projection
 * again; its workspace is morpho_sm100_backward_saved_workspace_size(p) bytes.  `saved`
 * must come from a forward_save call with the same problem, inputs and weights, and stay
 * untouched in between.  Results are bit-identical to forward + backward. */
MORPHO_API size_t morpho_sm100_saved_bytes(const morpho_problem_t* p);
MORPHO_API size_t morpho_sm100_backward_saved_workspace_size(const morpho_problem_t* p);
MORPHO_API int morpho_sm100_forward_save(const morpho_problem_t* p, const void* X, const void* W_phi,
                                         const void* gate_q, const void* gate_k, const void* W_V, void* out,
                                         float* lse, void* saved, size_t saved_bytes, void* stream);
MORPHO_API int morpho_sm100_backward_saved(const morpho_problem_t* p, const void* grad_out, const void* saved,
                                           size_t saved_bytes, const void* X, const void* W_phi,
                                           const void* gate_q, const void* gate_k, const void* W_V,
                                           const void* out, const float* lse, void* dX, void* dW_phi,
                                           void* d_gate_q, void* d_gate_k, void* dW_V, float* dweights_f32,
                                           void* workspace, size_t workspace_bytes, void* stream);

/* Data-parallel form of morpho_sm100_backward_saved (no reference counterpart: the reference
 * has no multi-GPU code): the weight gradients go to the fp32 bucket dweights_f32 (required),
 * which is complete before dX is computed; if bucket_ready (a cudaEvent_t) is non-NULL it is
 * recorded on the stream at that point, so the caller can all-reduce the bucket on another
 * stream while the dX GEMM runs, then call morpho_sm100_finalize_weight_grads.  Results are
 * bit-identical to morpho_sm100_backward_saved with the same bucket. */
MORPHO_API int morpho_sm100_backward_saved_dp(const morpho_problem_t* p, const void* grad_out, const void* saved,
                                              size_t saved_bytes, const void* X, const void* W_phi,
                                              const void* gate_q, const void* gate_k, const void* W_V,
                                              const void* out, const float* lse, void* dX, float* dweights_f32,
                                              void* bucket_ready, void* workspace, size_t workspace_bytes,
                                              void* stream);

/* Forward that allocates nothing, for callers that cannot allocate device memory where
 * they run it (a memory-pressure callback, a server whose memory plan is frozen after
 * start-up, a host language without an allocator binding).  No counterpart in the
 * reference.  Same arguments and results as morpho_sm100_forward minus the workspace: the
 * scratch lives in a fixed device array inside this library (size given by
 * morpho_sm100_forward_noalloc_max_scratch(), 32 MiB), held by every GPU that loads the
 * library until exit.  Problems whose forward workspace exceeds it are rejected with
 * MORPHO_ERR_WORKSPACE.  The first call on each device looks the array's address up
 * (cudaGetSymbolAddress); under CUDA's default lazy module loading that first call also
 * places the array and the forward's kernels on the device, so it reserves device memory:
 * make it at start-up, before the code that must not allocate, and outside any stream
 * capture.  Later calls reserve nothing.  Not usable again after cudaDeviceReset in the
 * same process.  All calls share the array: calls that overlap on the GPU race; calls
 * ordered on one stream are safe. */
MORPHO_API int morpho_sm100_forward_noalloc(const morpho_problem_t* p, const void* X, const void* W_phi,
                                            const void* gate_q, const void* gate_k, const void* W_V, void* out,
                                            float* lse, void* stream);
MORPHO_API size_t morpho_sm100_forward_noalloc_max_scratch(void);

/* Projection only (one GEMM with a fused epilogue): the per-head hypercube codes and
 * values the attention kernels consume.  Replaces the per-tile project_phi
 * (packages/morphottention/csrc/cuda/sm120/project.cuh:16-47) and the value projection
 * (attention.cu:106-111), which the reference recomputes for every query block.
 * Outputs, with BH = B*H and Npad = N rounded up to a multiple of 128:
 *   qc      fp16 [BH, N, cube_m]   gate_q*(phi - 1/2), phi = sigmoid(X @ W_phi_h): centered
 *                                  query codes, so kc . qc = q.k - cbias/2 (the column bias)
 *   kc      fp16 [BH, N, cube_m]   gate_k*phi
 *   v       fp16 [BH, N, D/H]      X @ W_V_h
 *   qb, cb  fp32 [BH, Npad]        scale*log2(e) * sum_c gate_k q_c, resp. sum_c gate_q k_c
 *   phi     fp32 [BH, N, cube_m]   optional (may be NULL)
 * All buffers 16-byte aligned. */
MORPHO_API int morpho_sm100_project(const morpho_problem_t* p, const void* X, const void* W_phi, const void* gate_q,
                                    const void* gate_k, const void* W_V, void* qc, void* kc, void* v, float* qb,
                                    float* cb, float* phi, void* stream);

/* Number of fp32 elements of the dweights_f32 bucket for problem p (one more, dL/dtau, for the
 * DILATION / EROSION scores). */
MORPHO_API size_t morpho_sm100_weight_grad_elems(const morpho_problem_t* p);

/* fp16 weight gradients = alpha * bucket (alpha = 1/world for a mean); the bucket's dL/dtau
 * element, if any, is left as it is.  No reference counterpart: the reference has no
 * data-parallel path. */
MORPHO_API int morpho_sm100_finalize_weight_grads(const morpho_problem_t* p, const float* dweights_f32, float alpha,
                                       void* dW_phi, void* d_gate_q, void* d_gate_k, void* dW_V, void* stream);

/* Peer-memory all-reduce of the data-parallel bucket, fused with the finalize (no reference
 * counterpart: the reference has no multi-GPU code).  One process per GPU of one node, every
 * pair of GPUs with peer access.  Each rank creates a group (its exchange region: a signal
 * block and two buckets of bucket_elems fp32, zero-filled, in its own device memory, exported
 * as a CUDA IPC handle of MORPHO_PEER_HANDLE_BYTES and identified by its GPU's PCI bus id, a
 * string of at most MORPHO_PEER_PCI_ID_BYTES), the caller exchanges the handles and ids between
 * the ranks (in rank order, world entries each) and every rank connects.  Per step: the
 * backward writes morpho_sm100_peer_bucket(g) -- the bucket of the next all-reduce, alternating
 * between the two -- then morpho_sm100_peer_allreduce_finalize enqueues ONE kernel on `stream`
 * that sums the ranks' buckets over NVLink (reduce-scatter, then all-gather, each rank summing
 * in rank order 0..world-1, so every rank gets the same bits), leaves the sum in that bucket and
 * writes the fp16 gradients alpha * sum, as morpho_sm100_finalize_weight_grads does.  Every rank
 * must call it the same number of times, and its stream must have waited for the bucket to be
 * complete.  The kernel needs no SM of its own (no shared memory): it runs beside a concurrent
 * kernel such as the dX GEMM.  Its waits for the other ranks are bounded (1 s); on expiry it
 * records MORPHO_ERR_TIMEOUT in the device status word and the group must be destroyed.
 * Destroy only when no rank can still be in an all-reduce (after a barrier).  connect returns
 * MORPHO_ERR_UNSUPPORTED when a peer's GPU is not visible or not peer-accessible (use NCCL). */
#define MORPHO_PEER_HANDLE_BYTES 64
#define MORPHO_PEER_PCI_ID_BYTES 32
typedef struct morpho_peer_group morpho_peer_group_t;
MORPHO_API int morpho_sm100_peer_create(int32_t rank, int32_t world, int64_t bucket_elems, void* handle_out,
                                        char* pci_bus_id_out, morpho_peer_group_t** group);
MORPHO_API int morpho_sm100_peer_connect(morpho_peer_group_t* group, const void* handles, const char* pci_bus_ids);
MORPHO_API float* morpho_sm100_peer_bucket(const morpho_peer_group_t* group);
MORPHO_API int morpho_sm100_peer_allreduce_finalize(morpho_peer_group_t* group, const morpho_problem_t* p,
                                                    float alpha, void* dW_phi, void* d_gate_q, void* d_gate_k,
                                                    void* dW_V, void* stream);
MORPHO_API int morpho_sm100_peer_destroy(morpho_peer_group_t* group);

/* Message of the last failure on the calling thread ("" if none). */
MORPHO_API const char* morpho_sm100_last_error(void);

/* Device status word of the current device: 0 when every bounded wait of every kernel
 * finished in time, else a code naming the kernel and wait that expired.  Synchronises
 * the stream.  reset != 0 clears the word after reading it. */
MORPHO_API int morpho_sm100_device_status(void* stream, int reset, uint32_t* status_out);

/* Failure-path self test (no reference counterpart): launches one kernel whose bounded wait
 * on a barrier that nothing arrives at gives up after limit_us microseconds (<= 1 s),
 * records its code (kernel 15, site 1, bit 31) in the device status word and returns.  Read
 * the word with morpho_sm100_device_status. */
MORPHO_API int morpho_sm100_selftest_wait_timeout(uint32_t limit_us, void* stream);

/* Design probe (no reference counterpart): the score the attention kernels issue as tcgen05
 * MMAs, computed instead on packed half2 CUDA-core math -- for every query row of every (batch,
 * head) the maximum over all keys of qc_i . k_j (cube_m/2 HFMA2 per pair, fp16 accumulation,
 * HMNMX2 row maxima).  qc, kc: fp16 [BH, N, cube_m] (the layouts of morpho_sm100_project);
 * rowmax: fp32 [BH, N].  Used to measure that alternative against the tensor-core kernels. */
MORPHO_API int morpho_sm100_score_probe_half2(const void* qc, const void* kc, int32_t BH, int32_t N, int32_t cube_m,
                                              float* rowmax, void* stream);

/* Number of kernels the last forward / backward call on this thread launched. */
MORPHO_API int morpho_sm100_last_launch_count(void);

/* Per-kernel timing for benchmarks (no reference counterpart).  While enabled, every
 * launch of this library records a CUDA event pair on its stream.  collect() waits for
 * the recorded events, writes up to max_kernels entries (kernel name into
 * names[i*name_len], summed milliseconds, launch count), clears the records and returns
 * the number of entries.  Process-wide switch; records are kept per host thread. */
MORPHO_API void morpho_sm100_profile_enable(int on);
MORPHO_API int morpho_sm100_profile_collect(char* names, int name_len, float* total_ms, int* counts,
                                            int max_kernels);
/* Restrict the timing to the launches of one kernel (the name collect() reports, e.g. "attn_bwd"):
 * the others record no events, so they run as they do unprofiled.  NULL or "" times every launch. */
MORPHO_API void morpho_sm100_profile_select(const char* kernel_name);

#ifdef __cplusplus
}
#endif

#endif /* MORPHO_SM100_H */
