// kernels.h -- internal launcher interface between the C ABI (capi.cu) and the sm_100a
// kernels (gemm.cu, attn_fwd.cu, attn_bwd.cu, pointwise.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "host_common.h"

namespace morpho {

constexpr float kLog2e = 1.4426950408889634f;

// Hypercube projections (the values of MORPHO_PROJ_* in morpho_sm100.h).
constexpr int kProjSigmoid = 0;
constexpr int kProjHardTanh01 = 1;
constexpr int kProjIdentity = 2;
// Scores (the values of MORPHO_SCORE_*).
constexpr int kScoreSoftmax = 0;
constexpr int kScoreDilation = 1;
constexpr int kScoreErosion = 2;

struct Shape {
    int B, N, D, H, m, hd;
    float scale;
    bool causal;
    int grad_mode;
    int proj = 0;            // MORPHO_PROJ_*
    bool mask_diag = false;  // drop key j == query i
    int score = 0;           // kScore*
    float tau = 1.0f;        // soft-morphology temperature
    long long tokens() const { return static_cast<long long>(B) * N; }
    int Hm() const { return H * m; }
    // dZ columns are padded to a multiple of 64 so that no 64-wide K block of the dX
    // GEMM straddles W_phi and W_V; the pad columns of dcat hold zeros.
    int Hp() const { return (H * m + 63) / 64 * 64; }
    int Cp() const { return Hp() + D; }  // width of dcat = [dZ | 0 | dV]
};

// Per-(b, h) intermediates written by the projection GEMM epilogue.  Head-major so an
// attention tile is one contiguous box: codes [B*H, N, m], V [B*H, N, hd], biases
// [B*H, N] pre-multiplied by scale*log2(e).
struct ProjOut {
    // Centered query codes gate_q * (phi - 1/2).  Since cb_j = sum_c gate_q,c k_jc, the
    // plain dot product k_j . qc_i equals k_j . q_i - cb_j / 2: the score MMA yields the
    // column-biased score directly, and dK = dS^T . qc needs no cancelling bias term.
    __half* qc = nullptr;
    __half* kc = nullptr;   // gate_k * phi
    __half* v = nullptr;    // x @ W_V head slice
    float* qb = nullptr;    // scale*log2e * sum_c gate_k q_c
    float* cb = nullptr;    // scale*log2e * sum_c gate_q k_c
    float* phi = nullptr;   // optional fp32 phi [B*H, N, m] (backward recompute)
    // Optional (backward): centered key codes k - gate_k/2 split into fp16 hi + lo parts,
    // interleaved per row as [hi (m) | lo (m)], [B*H, N, 2m].  dq = dS . k is computed as
    // dS . hi + dS . lo: every row of dS sums to zero, so the centering term drops out
    // exactly while the fp16 rounding of the large mean of k no longer leaks into dq.
    __half* kdq = nullptr;
    // Soft-morphology score (training pair / backward only): m + log2(l) per (row, channel),
    // fp32 [B*H, N, hd], written by the forward for the backward.
    float* o2 = nullptr;
    // Soft-morphology tensor-core forward scratch: E_V^T [B*H, hd, Npad] fp32, R [B*H, hd],
    // per-256-key column maxima [B*H, ceil(N/256), hd], and the fallback flag.
    float* evt = nullptr;
    float* rv = nullptr;
    float* vpart = nullptr;
    uint32_t* smflag = nullptr;
    float* mrow = nullptr;  // [B*H, Npad] the split forward's row reference m_i
};

// X [T, D] @ [W_phi | W_V] with the sigmoid / gating / bias epilogue.
int launch_proj(const DeviceInfo& dev, const Shape& s, const __half* X, const __half* W_phi, const __half* W_V,
                const __half* gate_q, const __half* gate_k, const ProjOut& o, cudaStream_t stream);

// dX [T, D] = dcat [T, Cp] @ [W_phi | 0 | W_V]^T.
int launch_dx(const DeviceInfo& dev, const Shape& s, const __half* dcat, const __half* W_phi, const __half* W_V,
              __half* dX, cudaStream_t stream);

// part[z] [D, Cp] = X^T [D, T] @ dcat [T, Cp] over the z-th slice of tokens.
int launch_dw(const DeviceInfo& dev, const Shape& s, const __half* X, const __half* dcat, float* part, int splits,
              cudaStream_t stream);
int dw_splits(const DeviceInfo& dev, const Shape& s);

// Attention forward over the projected codes: out fp16 [B, N, D], lse fp32 [B*H, N].
int launch_attn_fwd(const DeviceInfo& dev, const Shape& s, const ProjOut& p, __half* out, float* lse,
                    cudaStream_t stream);

// Attention backward (KV-stationary).  Inputs: codes/V/bias slices, dO, L = lse + qb
// (log2 domain, without the query bias), the query slice qaug.  Outputs: dV into
// dcat[:, Hp + h*hd + e] (fp16), dk (fp32 [B*H, N, m], = 2*scale * dS^T qc with the
// centered query codes),
// dcb (fp32 [B*H, N], = -scale * sum_i dS_ij), and dq (fp32 [B*H, N, m], accumulated
// with atomics, = 2*scale * dS k; must be zeroed first).
struct AttnBwdIO {
    const __half* dO;
    const float* L;
    const __half* qaug;
    __half* dcat;
    float* dk;
    float* dcb;
    float* dq;
};
int launch_attn_bwd(const DeviceInfo& dev, const Shape& s, const ProjOut& p, const AttnBwdIO& io,
                    cudaStream_t stream);

// Per query row (padded [B*H, Npad] fp32) L = lse + qb, and the query slice of the
// augmented backward MMAs, fp16 [B*H, N, 16]: [1, 1, -delta (hi), -delta (lo), 0 ...] with
// delta = sum_e dO * O over the head slice (attention.cu:294-311).
int launch_delta(const Shape& s, const __half* dO, const __half* O, const float* lse, const float* qb, float* L,
                 __half* qaug, cudaStream_t stream);

// dZ = dL/dphi * phi (1 - phi) into dcat[:, h*m + c] and per-block gate partials.
// Soft-morphology score (softmorph.cu): forward out (fp16, may be NULL) and o2 = m + log2(l)
// per (row, channel) [B*H, N, hd] fp32 (may be NULL); backward dq, dqb ([B*H, Npad]), dk, dcb
// and the dV columns of dcat from the forward's o2.
// Exact CUDA-core forward; with only_if set it runs only when *only_if != 0 (device-side).
int launch_soft_morph_fwd(const Shape& s, const ProjOut& p, __half* out, float* o2, const uint32_t* only_if,
                          cudaStream_t stream);
// Soft-morphology path choice: the environment variable MORPHO_SOFT_MORPH_EXACT (set and not
// "0") selects the exact CUDA-core kernels only; otherwise the split (tensor-core forward and
// backward) runs, guarded by the exact kernels.
bool soft_morph_exact_only();
// Tensor-core forward (E_S . E_V split) followed by the exact forward as its guard.
int launch_soft_morph_fwd_tc(const DeviceInfo& dev, const Shape& s, const ProjOut& p, __half* out, float* o2,
                             cudaStream_t stream);
// fp32 operand layouts of the tensor-core soft-morphology backward (every head dim):
// G [B*H, N, hd], G^T [B*H, hd, Npad], E_V [B*H, Npad, hd], kd^T and qc^T [B*H, m, Npad].
struct SmBwdScratch {
    float* g = nullptr;
    float* gt = nullptr;
    float* evn = nullptr;
    float* kdt = nullptr;
    float* qct = nullptr;
};
int launch_soft_morph_bwd_tc(const Shape& s, const ProjOut& p, const SmBwdScratch& x, const __half* dO,
                             const float* o2, float* dq, float* dqb, float* sg, float* dk, float* dcb,
                             __half* dcat, uint32_t* status, cudaStream_t stream);
// Soft-morphology backward: the tensor-core split kernels and, gated against them by the forward's
// range flag, the exact kernels; the exact kernels alone under the MORPHO_SOFT_MORPH_EXACT switch.
// sg (may be NULL): per query row sum_j S_ij dL/dS_ij [B*H, Npad], for the temperature gradient.
int launch_soft_morph_bwd(const Shape& s, const ProjOut& p, const SmBwdScratch* tcx, uint32_t* status,
                          const __half* dO, const float* o2, float* dq, float* dqb, float* sg,
                          float* dk, float* dcb, __half* dcat, cudaStream_t stream);
// dL/dtau of the soft-morphology score into *dtau (device fp32), after launch_soft_morph_bwd left
// sg and the dV columns of dcat; part holds soft_morph_dtau_parts(s) floats of partial sums.
size_t soft_morph_dtau_parts(const Shape& s);
int launch_soft_morph_dtau(const Shape& s, const ProjOut& p, const __half* dO, const float* o2, const float* sg,
                           const __half* dcat, float* part, float* dtau, cudaStream_t stream);

// dqb (dL/dqbias, [B*H, Npad]) may be NULL: the softmax score's rows are shift-invariant, so
// its query-bias gradient is identically 0.
int launch_dz(const Shape& s, const float* phi, const float* dq, const float* dk, const float* dcb,
              const float* dqb, const __half* gate_q, const __half* gate_k, __half* dcat, float* gate_part,
              int gate_blocks, cudaStream_t stream);
int dz_gate_blocks(const Shape& s);

// Sum the dW split partials and gate partials: either into an fp32 bucket (layout of
// morpho_sm100_backward's dweights_f32) or straight to fp16 outputs.
int launch_reduce_weights(const Shape& s, const float* dw_part, int splits, const float* gate_part, int gate_blocks,
                          float* bucket, __half* dW_phi, __half* dW_V, __half* d_gate_q, __half* d_gate_k,
                          cudaStream_t stream);

// Band width of the causal launch order (causal_order in sm100.cuh): 1 (longest first) when the
// BH streams of `bytes_per_bh` each fit comfortably in L2 together; else all n_t tiles of a
// (batch, head) in turn, so that the CTAs running together share few streams (at c5, bands of 8
// tiles were 1.5 % slower than this, from the extra L2 misses, although they shorten the tail).
inline int causal_band(long long bytes_per_bh, int BH, int n_t) {
    return bytes_per_bh * BH <= (48ll << 20) ? 1 : n_t;
}

// fp16 outputs = alpha * bucket.
int launch_finalize_weights(const Shape& s, const float* bucket, float alpha, __half* dW_phi, __half* dW_V,
                            __half* d_gate_q, __half* d_gate_k, cudaStream_t stream);

}  // namespace morpho
