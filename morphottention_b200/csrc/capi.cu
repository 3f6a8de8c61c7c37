// capi.cu -- the extern "C" entry points of libmorpho_sm100.so (declared in
// include/morpho_sm100.h): argument validation, workspace planning and the kernel
// sequence of the forward and backward passes.
//
// Forward  (2 launches): projection GEMM+epilogue -> attention forward.
// Backward (7 launches + 1 memset): projection recompute (+phi) -> delta/L ->
//   zero dq -> attention backward -> dZ + gate partials -> dW GEMM (split-K) ->
//   deterministic reduction of dW / gate partials -> dX GEMM.
#include <string.h>

#include "kernels.h"

using namespace morpho;

namespace {

constexpr int kTile = 128;
static_assert(kProjSigmoid == MORPHO_PROJ_SIGMOID && kProjHardTanh01 == MORPHO_PROJ_HARDTANH01 &&
                  kProjIdentity == MORPHO_PROJ_IDENTITY,
              "projection codes");
static_assert(kScoreSoftmax == MORPHO_SCORE_SOFTMAX && kScoreDilation == MORPHO_SCORE_DILATION &&
                  kScoreErosion == MORPHO_SCORE_EROSION,
              "score codes");

int validate(const morpho_problem_t* p, Shape* s) {
    if (p == nullptr) return set_error(MORPHO_ERR_INVALID, "problem is NULL");
    if (p->B <= 0 || p->N <= 0 || p->D <= 0 || p->H <= 0)
        return set_error(MORPHO_ERR_INVALID, "Invalid dimensions: B=%d N=%d D=%d H=%d", p->B, p->N, p->D, p->H);
    if (p->D % p->H != 0) return set_error(MORPHO_ERR_INVALID, "D must be divisible by H (D=%d, H=%d)", p->D, p->H);
    const int hd = p->D / p->H;
    if (hd != 32 && hd != 64 && hd != 128)
        return set_error(MORPHO_ERR_INVALID, "head_dim D/H = %d not supported (32, 64 or 128)", hd);
    if (p->cube_m != 16 && p->cube_m != 32 && p->cube_m != 64)
        return set_error(MORPHO_ERR_INVALID, "cube_m = %d not supported (16, 32 or 64)", p->cube_m);
    if (p->grad_mode != MORPHO_GRAD_FULL && p->grad_mode != MORPHO_GRAD_REFERENCE)
        return set_error(MORPHO_ERR_INVALID, "grad_mode %d unknown", p->grad_mode);
    if (p->projection != MORPHO_PROJ_SIGMOID && p->projection != MORPHO_PROJ_HARDTANH01 &&
        p->projection != MORPHO_PROJ_IDENTITY)
        return set_error(MORPHO_ERR_INVALID, "projection %d unknown", p->projection);
    if (p->mask_diag != 0 && p->mask_diag != 1)
        return set_error(MORPHO_ERR_INVALID, "mask_diag must be 0 or 1 (got %d)", p->mask_diag);
    if (p->score != MORPHO_SCORE_SOFTMAX && p->score != MORPHO_SCORE_DILATION && p->score != MORPHO_SCORE_EROSION)
        return set_error(MORPHO_ERR_INVALID, "score %d unknown", p->score);
    if (p->score != MORPHO_SCORE_SOFTMAX) {
        if (!(p->tau > 0.0f) || p->tau > 1e30f)
            return set_error(MORPHO_ERR_INVALID, "tau must be positive and finite (got %g)", static_cast<double>(p->tau));
        if (p->grad_mode != MORPHO_GRAD_FULL)
            return set_error(MORPHO_ERR_INVALID, "grad_mode reference applies to the softmax score only");
    }
    const long long T = static_cast<long long>(p->B) * p->N;
    if (T > (1LL << 30) || static_cast<long long>(p->B) * p->H * p->N * 128 > (1LL << 40))
        return set_error(MORPHO_ERR_INVALID, "problem too large: B*N = %lld", T);
    if (static_cast<long long>(p->B) * p->H > 65535)
        return set_error(MORPHO_ERR_INVALID, "B*H = %lld exceeds the grid limit 65535",
                         static_cast<long long>(p->B) * p->H);
    s->B = p->B;
    s->N = p->N;
    s->D = p->D;
    s->H = p->H;
    s->m = p->cube_m;
    s->hd = hd;
    s->scale = p->scale;
    s->causal = p->causal != 0;
    s->grad_mode = p->grad_mode;
    s->proj = p->projection;
    s->mask_diag = p->mask_diag != 0;
    s->score = p->score;
    s->tau = p->tau;
    return MORPHO_OK;
}

// The attention step of the forward: softmax . V, or the soft-morphology aggregation (which
// has no lse: 0 is written).
int run_attention_fwd(const DeviceInfo& dev, const Shape& s, const ProjOut& proj, __half* out, float* lse,
                      cudaStream_t st) {
    if (s.score == kScoreSoftmax) return launch_attn_fwd(dev, s, proj, out, lse, st);
    MORPHO_CUDA_TRY(cudaMemsetAsync(lse, 0, static_cast<size_t>(s.B) * s.H * s.N * sizeof(float), st));
    return launch_soft_morph_fwd_tc(dev, s, proj, out, proj.o2, st);  // o2 kept by forward_save only
}

int check_ptr(const void* ptr, const char* name) {
    if (ptr == nullptr) return set_error(MORPHO_ERR_INVALID, "%s is NULL", name);
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0)
        return set_error(MORPHO_ERR_INVALID, "%s is not 16-byte aligned", name);
    return MORPHO_OK;
}

// Bump allocator over the caller's workspace (256-byte aligned sub-buffers).
struct Carve {
    uint8_t* base;
    size_t off = 0;
    explicit Carve(void* b) : base(static_cast<uint8_t*>(b)) {}
    template <class T>
    T* take(size_t count) {
        off = (off + 255) / 256 * 256;
        T* ptr = base ? reinterpret_cast<T*>(base + off) : nullptr;
        off += count * sizeof(T);
        return ptr;
    }
};

struct FwdPlan {
    ProjOut proj;
};

void plan_proj(Carve& c, const Shape& s, ProjOut* o) {
    const size_t BH = static_cast<size_t>(s.B) * s.H;
    const size_t Npad = (s.N + kTile - 1) / kTile * kTile;
    o->qc = c.take<__half>(BH * s.N * s.m);
    o->kc = c.take<__half>(BH * s.N * s.m);
    o->v = c.take<__half>(BH * s.N * s.hd);
    o->qb = c.take<float>(BH * Npad);
    o->cb = c.take<float>(BH * Npad);
    if (s.score != kScoreSoftmax) {
        o->evt = c.take<float>(BH * s.hd * Npad);
        o->rv = c.take<float>(BH * s.hd);
        o->vpart = c.take<float>(BH * ((s.N + 255) / 256) * s.hd);
        o->smflag = c.take<uint32_t>(64);
        o->mrow = c.take<float>(BH * Npad);
    }
}

struct BwdPlan {
    ProjOut proj;
    __half* qaug;
    float* L;
    float* dqb;  // soft-morphology score: dL/dqbias, [B*H, Npad]
    float* sg;         // soft-morphology score: sum_j S_ij dL/dS_ij per query row, [B*H, Npad]
    float* dtau_part;  // soft-morphology score: partial sums of dL/dtau
    SmBwdScratch smx;  // soft-morphology tensor-core backward operands
    float* dq;
    float* dk;
    float* dcb;
    __half* dcat;
    float* dw_part;
    float* gate_part;
    int splits;
    int gate_blocks;
};

// Every projection output the backward reads (what forward_save keeps).
void plan_saved(Carve& c, const Shape& s, ProjOut* o) {
    const size_t BH = static_cast<size_t>(s.B) * s.H;
    plan_proj(c, s, o);
    o->phi = c.take<float>(BH * s.N * s.m);
    o->kdq = c.take<__half>(BH * s.N * 2 * s.m);
    o->o2 = s.score != kScoreSoftmax ? c.take<float>(BH * s.N * s.hd) : nullptr;
}

// The backward's own buffers, after the projection outputs.
void plan_bwd_rest(Carve& c, const Shape& s, int sms, BwdPlan* b) {
    const size_t BH = static_cast<size_t>(s.B) * s.H;
    const size_t Npad = (s.N + kTile - 1) / kTile * kTile;
    b->qaug = c.take<__half>(BH * s.N * 16);
    b->L = c.take<float>(BH * Npad);
    b->dqb = s.score != kScoreSoftmax ? c.take<float>(BH * Npad) : nullptr;
    b->sg = s.score != kScoreSoftmax ? c.take<float>(BH * Npad) : nullptr;
    b->dtau_part = s.score != kScoreSoftmax ? c.take<float>(soft_morph_dtau_parts(s)) : nullptr;
    if (s.score != kScoreSoftmax) {
        b->smx.g = c.take<float>(BH * s.N * s.hd);
        b->smx.gt = c.take<float>(BH * s.hd * Npad);
        b->smx.evn = c.take<float>(BH * Npad * s.hd);
        b->smx.kdt = c.take<float>(BH * s.m * Npad);
        b->smx.qct = c.take<float>(BH * s.m * Npad);
    }
    b->dq = c.take<float>(BH * s.N * s.m);
    b->dk = c.take<float>(BH * s.N * s.m);
    b->dcb = c.take<float>(BH * Npad);
    b->dcat = c.take<__half>(static_cast<size_t>(s.tokens()) * s.Cp());
    DeviceInfo d;
    d.sms = sms;
    b->splits = dw_splits(d, s);
    b->dw_part = c.take<float>(static_cast<size_t>(b->splits) * s.D * s.Cp());
    b->gate_blocks = dz_gate_blocks(s);
    b->gate_part = c.take<float>(static_cast<size_t>(b->gate_blocks) * 2 * s.Hm());
}

void plan_bwd(Carve& c, const Shape& s, int sms, BwdPlan* b) {
    plan_saved(c, s, &b->proj);
    plan_bwd_rest(c, s, sms, b);
}

// Argument checks shared by both backward entry points.
int check_bwd_args(const void* grad_out, const void* X, const void* W_phi, const void* gate_q, const void* gate_k,
                   const void* W_V, const void* out, const float* lse, void* dX, void* dW_phi, void* d_gate_q,
                   void* d_gate_k, void* dW_V, float* dweights_f32, void* workspace) {
    MORPHO_TRY(check_ptr(grad_out, "grad_out"));
    MORPHO_TRY(check_ptr(X, "X"));
    MORPHO_TRY(check_ptr(W_phi, "W_phi"));
    MORPHO_TRY(check_ptr(gate_q, "gate_q"));
    MORPHO_TRY(check_ptr(gate_k, "gate_k"));
    MORPHO_TRY(check_ptr(W_V, "W_V"));
    MORPHO_TRY(check_ptr(out, "out"));
    MORPHO_TRY(check_ptr(lse, "lse"));
    MORPHO_TRY(check_ptr(dX, "dX"));
    if (dweights_f32 != nullptr) {
        MORPHO_TRY(check_ptr(dweights_f32, "dweights_f32"));
    } else {
        MORPHO_TRY(check_ptr(dW_phi, "dW_phi"));
        MORPHO_TRY(check_ptr(d_gate_q, "d_gate_q"));
        MORPHO_TRY(check_ptr(d_gate_k, "d_gate_k"));
        MORPHO_TRY(check_ptr(dW_V, "dW_V"));
    }
    MORPHO_TRY(check_ptr(workspace, "workspace"));
    return MORPHO_OK;
}

// Elements of the fp32 weight-gradient bucket before the optional dL/dtau:
// [dW_phi | dW_V | d_gate_q | d_gate_k].
size_t weight_elems(const Shape& s) {
    return static_cast<size_t>(s.D) * (s.Hm() + s.D) + 2u * static_cast<size_t>(s.Hm());
}

// Everything of the backward after the projection: delta, attention backward, the
// sigmoid/gate chain rule, the weight-gradient chain (dW GEMM, reduction) and then the dX
// GEMM, so that a data-parallel caller can start the all-reduce of the weight gradients
// (bucket_ready, recorded in between) while dX runs.
int run_backward_after_proj(const DeviceInfo& dev, const Shape& s, const BwdPlan& b, const void* grad_out,
                            const void* X, const void* W_phi, const void* gate_q, const void* gate_k,
                            const void* W_V, const void* out, const float* lse, void* dX, void* dW_phi,
                            void* d_gate_q, void* d_gate_k, void* dW_V, float* dweights_f32, cudaStream_t st,
                            cudaEvent_t bucket_ready = nullptr, bool o2_ready = false) {
    const __half* x = static_cast<const __half*>(X);
    const __half* wphi = static_cast<const __half*>(W_phi);
    const __half* wv = static_cast<const __half*>(W_V);
    const __half* gq = static_cast<const __half*>(gate_q);
    const __half* gk = static_cast<const __half*>(gate_k);
    if (s.score == kScoreSoftmax) {
        MORPHO_TRY(launch_delta(s, static_cast<const __half*>(grad_out), static_cast<const __half*>(out), lse,
                                b.proj.qb, b.L, b.qaug, st));
        MORPHO_CUDA_TRY(cudaMemsetAsync(b.dq, 0, static_cast<size_t>(s.B) * s.H * s.N * s.m * sizeof(float), st));
        AttnBwdIO io;
        io.dO = static_cast<const __half*>(grad_out);
        io.L = b.L;
        io.qaug = b.qaug;
        io.dcat = b.dcat;
        io.dk = b.dk;
        io.dcb = b.dcb;
        io.dq = b.dq;
        MORPHO_TRY(launch_attn_bwd(dev, s, b.proj, io, st));
    } else {
        // soft-morphology score: the forward's m + log2(l) (kept by forward_save, else
        // recomputed), then the two backward kernels
        if (!o2_ready) MORPHO_TRY(launch_soft_morph_fwd_tc(dev, s, b.proj, nullptr, b.proj.o2, st));
        // the temperature gradient goes to the bucket's last element (no fp16 form)
        float* dtau = dweights_f32 != nullptr ? dweights_f32 + weight_elems(s) : nullptr;
        MORPHO_TRY(launch_soft_morph_bwd(s, b.proj, b.smx.g != nullptr ? &b.smx : nullptr, dev.status,
                                         static_cast<const __half*>(grad_out), b.proj.o2, b.dq, b.dqb,
                                         dtau != nullptr ? b.sg : nullptr, b.dk, b.dcb, b.dcat, st));
        if (dtau != nullptr)
            MORPHO_TRY(launch_soft_morph_dtau(s, b.proj, static_cast<const __half*>(grad_out), b.proj.o2, b.sg,
                                              b.dcat, b.dtau_part, dtau, st));
    }
    MORPHO_TRY(launch_dz(s, b.proj.phi, b.dq, b.dk, b.dcb, b.dqb, gq, gk, b.dcat, b.gate_part, b.gate_blocks, st));
    MORPHO_TRY(launch_dw(dev, s, x, b.dcat, b.dw_part, b.splits, st));
    MORPHO_TRY(launch_reduce_weights(s, b.dw_part, b.splits, b.gate_part, b.gate_blocks, dweights_f32,
                                     static_cast<__half*>(dW_phi), static_cast<__half*>(dW_V),
                                     static_cast<__half*>(d_gate_q), static_cast<__half*>(d_gate_k), st));
    if (bucket_ready != nullptr) MORPHO_CUDA_TRY(cudaEventRecord(bucket_ready, st));
    MORPHO_TRY(launch_dx(dev, s, b.dcat, wphi, wv, static_cast<__half*>(dX), st));
    return MORPHO_OK;
}

// The workspace size depends on the SM count (split-K factor); query the current
// device when there is one, else assume a full B200.
int sms_for_sizing() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) ==
                                                  cudaSuccess && sms > 0)
        return sms;
    cudaGetLastError();
    return 148;
}

}  // namespace

extern "C" {

size_t morpho_sm100_forward_workspace_size(const morpho_problem_t* p) {
    Shape s;
    if (validate(p, &s) != MORPHO_OK) return 0;
    Carve c(nullptr);
    FwdPlan f;
    plan_proj(c, s, &f.proj);
    return c.off + 256;
}

size_t morpho_sm100_backward_workspace_size(const morpho_problem_t* p) {
    Shape s;
    if (validate(p, &s) != MORPHO_OK) return 0;
    Carve c(nullptr);
    BwdPlan b;
    plan_bwd(c, s, sms_for_sizing(), &b);
    return c.off + 256;
}

size_t morpho_sm100_weight_grad_elems(const morpho_problem_t* p) {
    Shape s;
    if (validate(p, &s) != MORPHO_OK) return 0;
    return weight_elems(s) + (s.score != kScoreSoftmax ? 1u : 0u);  // + dL/dtau
}

int morpho_sm100_forward(const morpho_problem_t* p, const void* X, const void* W_phi, const void* gate_q,
                         const void* gate_k, const void* W_V, void* out, float* lse, void* workspace,
                         size_t workspace_bytes, void* stream) {
    clear_error();
    reset_launch_count();
    Shape s;
    MORPHO_TRY(validate(p, &s));
    MORPHO_TRY(check_ptr(X, "X"));
    MORPHO_TRY(check_ptr(W_phi, "W_phi"));
    MORPHO_TRY(check_ptr(gate_q, "gate_q"));
    MORPHO_TRY(check_ptr(gate_k, "gate_k"));
    MORPHO_TRY(check_ptr(W_V, "W_V"));
    MORPHO_TRY(check_ptr(out, "out"));
    MORPHO_TRY(check_ptr(lse, "lse"));
    MORPHO_TRY(check_ptr(workspace, "workspace"));
    const size_t need = morpho_sm100_forward_workspace_size(p);
    if (workspace_bytes < need)
        return set_error(MORPHO_ERR_WORKSPACE, "forward workspace too small: %zu < %zu bytes", workspace_bytes, need);
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Carve c(workspace);
    FwdPlan f;
    plan_proj(c, s, &f.proj);
    const __half* x = static_cast<const __half*>(X);
    MORPHO_TRY(launch_proj(dev, s, x, static_cast<const __half*>(W_phi), static_cast<const __half*>(W_V),
                           static_cast<const __half*>(gate_q), static_cast<const __half*>(gate_k), f.proj, st));
    MORPHO_TRY(run_attention_fwd(dev, s, f.proj, static_cast<__half*>(out), lse, st));
    return MORPHO_OK;
}

int morpho_sm100_backward(const morpho_problem_t* p, const void* grad_out, const void* X, const void* W_phi,
                          const void* gate_q, const void* gate_k, const void* W_V, const void* out,
                          const float* lse, void* dX, void* dW_phi, void* d_gate_q, void* d_gate_k, void* dW_V,
                          float* dweights_f32, void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    reset_launch_count();
    Shape s;
    MORPHO_TRY(validate(p, &s));
    MORPHO_TRY(check_bwd_args(grad_out, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi, d_gate_q, d_gate_k,
                              dW_V, dweights_f32, workspace));
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    Carve need_c(nullptr);
    BwdPlan need_plan;
    plan_bwd(need_c, s, dev.sms, &need_plan);
    if (workspace_bytes < need_c.off + 256)
        return set_error(MORPHO_ERR_WORKSPACE, "backward workspace too small: %zu < %zu bytes", workspace_bytes,
                         need_c.off + 256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Carve c(workspace);
    BwdPlan b;
    plan_bwd(c, s, dev.sms, &b);
    MORPHO_TRY(launch_proj(dev, s, static_cast<const __half*>(X), static_cast<const __half*>(W_phi),
                           static_cast<const __half*>(W_V), static_cast<const __half*>(gate_q),
                           static_cast<const __half*>(gate_k), b.proj, st));
    return run_backward_after_proj(dev, s, b, grad_out, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi, d_gate_q,
                                   d_gate_k, dW_V, dweights_f32, st);
}

size_t morpho_sm100_saved_bytes(const morpho_problem_t* p) {
    Shape s;
    if (validate(p, &s) != MORPHO_OK) return 0;
    Carve c(nullptr);
    ProjOut o;
    plan_saved(c, s, &o);
    return c.off + 256;
}

size_t morpho_sm100_backward_saved_workspace_size(const morpho_problem_t* p) {
    Shape s;
    if (validate(p, &s) != MORPHO_OK) return 0;
    Carve c(nullptr);
    BwdPlan b;
    plan_bwd_rest(c, s, sms_for_sizing(), &b);
    return c.off + 256;
}

int morpho_sm100_forward_save(const morpho_problem_t* p, const void* X, const void* W_phi, const void* gate_q,
                              const void* gate_k, const void* W_V, void* out, float* lse, void* saved,
                              size_t saved_bytes, void* stream) {
    clear_error();
    reset_launch_count();
    Shape s;
    MORPHO_TRY(validate(p, &s));
    MORPHO_TRY(check_ptr(X, "X"));
    MORPHO_TRY(check_ptr(W_phi, "W_phi"));
    MORPHO_TRY(check_ptr(gate_q, "gate_q"));
    MORPHO_TRY(check_ptr(gate_k, "gate_k"));
    MORPHO_TRY(check_ptr(W_V, "W_V"));
    MORPHO_TRY(check_ptr(out, "out"));
    MORPHO_TRY(check_ptr(lse, "lse"));
    MORPHO_TRY(check_ptr(saved, "saved"));
    const size_t need = morpho_sm100_saved_bytes(p);
    if (saved_bytes < need)
        return set_error(MORPHO_ERR_WORKSPACE, "saved buffer too small: %zu < %zu bytes", saved_bytes, need);
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Carve c(saved);
    ProjOut o;
    plan_saved(c, s, &o);
    MORPHO_TRY(launch_proj(dev, s, static_cast<const __half*>(X), static_cast<const __half*>(W_phi),
                           static_cast<const __half*>(W_V), static_cast<const __half*>(gate_q),
                           static_cast<const __half*>(gate_k), o, st));
    MORPHO_TRY(run_attention_fwd(dev, s, o, static_cast<__half*>(out), lse, st));
    return MORPHO_OK;
}

namespace {
int backward_saved_impl(const morpho_problem_t* p, const void* grad_out, const void* saved, size_t saved_bytes,
                        const void* X, const void* W_phi, const void* gate_q, const void* gate_k, const void* W_V,
                        const void* out, const float* lse, void* dX, void* dW_phi, void* d_gate_q, void* d_gate_k,
                        void* dW_V, float* dweights_f32, void* bucket_ready, void* workspace, size_t workspace_bytes,
                        void* stream) {
    clear_error();
    reset_launch_count();
    Shape s;
    MORPHO_TRY(validate(p, &s));
    MORPHO_TRY(check_ptr(saved, "saved"));
    MORPHO_TRY(check_bwd_args(grad_out, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi, d_gate_q, d_gate_k,
                              dW_V, dweights_f32, workspace));
    if (saved_bytes < morpho_sm100_saved_bytes(p))
        return set_error(MORPHO_ERR_WORKSPACE, "saved buffer too small: %zu < %zu bytes", saved_bytes,
                         morpho_sm100_saved_bytes(p));
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    Carve need_c(nullptr);
    BwdPlan need_plan;
    plan_bwd_rest(need_c, s, dev.sms, &need_plan);
    if (workspace_bytes < need_c.off + 256)
        return set_error(MORPHO_ERR_WORKSPACE, "backward workspace too small: %zu < %zu bytes", workspace_bytes,
                         need_c.off + 256);
    Carve cs(const_cast<void*>(saved));
    BwdPlan b;
    plan_saved(cs, s, &b.proj);
    Carve c(workspace);
    plan_bwd_rest(c, s, dev.sms, &b);
    return run_backward_after_proj(dev, s, b, grad_out, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi, d_gate_q,
                                   d_gate_k, dW_V, dweights_f32, static_cast<cudaStream_t>(stream),
                                   static_cast<cudaEvent_t>(bucket_ready), /*o2_ready=*/true);
}
}  // namespace

int morpho_sm100_backward_saved(const morpho_problem_t* p, const void* grad_out, const void* saved,
                                size_t saved_bytes, const void* X, const void* W_phi, const void* gate_q,
                                const void* gate_k, const void* W_V, const void* out, const float* lse, void* dX,
                                void* dW_phi, void* d_gate_q, void* d_gate_k, void* dW_V, float* dweights_f32,
                                void* workspace, size_t workspace_bytes, void* stream) {
    return backward_saved_impl(p, grad_out, saved, saved_bytes, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi,
                               d_gate_q, d_gate_k, dW_V, dweights_f32, nullptr, workspace, workspace_bytes, stream);
}

int morpho_sm100_backward_saved_dp(const morpho_problem_t* p, const void* grad_out, const void* saved,
                                   size_t saved_bytes, const void* X, const void* W_phi, const void* gate_q,
                                   const void* gate_k, const void* W_V, const void* out, const float* lse, void* dX,
                                   float* dweights_f32, void* bucket_ready, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    if (dweights_f32 == nullptr) {
        clear_error();
        return set_error(MORPHO_ERR_INVALID, "dweights_f32 is NULL");
    }
    return backward_saved_impl(p, grad_out, saved, saved_bytes, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, nullptr,
                               nullptr, nullptr, nullptr, dweights_f32, bucket_ready, workspace, workspace_bytes,
                               stream);
}

int morpho_sm100_project(const morpho_problem_t* p, const void* X, const void* W_phi, const void* gate_q,
                         const void* gate_k, const void* W_V, void* qc, void* kc, void* v, float* qb, float* cb,
                         float* phi, void* stream) {
    clear_error();
    reset_launch_count();
    Shape s;
    MORPHO_TRY(validate(p, &s));
    MORPHO_TRY(check_ptr(X, "X"));
    MORPHO_TRY(check_ptr(W_phi, "W_phi"));
    MORPHO_TRY(check_ptr(gate_q, "gate_q"));
    MORPHO_TRY(check_ptr(gate_k, "gate_k"));
    MORPHO_TRY(check_ptr(W_V, "W_V"));
    MORPHO_TRY(check_ptr(qc, "qc"));
    MORPHO_TRY(check_ptr(kc, "kc"));
    MORPHO_TRY(check_ptr(v, "v"));
    MORPHO_TRY(check_ptr(qb, "qb"));
    MORPHO_TRY(check_ptr(cb, "cb"));
    if (phi != nullptr) MORPHO_TRY(check_ptr(phi, "phi"));
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    ProjOut o;
    o.qc = static_cast<__half*>(qc);
    o.kc = static_cast<__half*>(kc);
    o.v = static_cast<__half*>(v);
    o.qb = qb;
    o.cb = cb;
    o.phi = phi;
    return launch_proj(dev, s, static_cast<const __half*>(X), static_cast<const __half*>(W_phi),
                       static_cast<const __half*>(W_V), static_cast<const __half*>(gate_q),
                       static_cast<const __half*>(gate_k), o, static_cast<cudaStream_t>(stream));
}

int morpho_sm100_finalize_weight_grads(const morpho_problem_t* p, const float* dweights_f32, float alpha,
                                       void* dW_phi, void* d_gate_q, void* d_gate_k, void* dW_V, void* stream) {
    clear_error();
    reset_launch_count();
    Shape s;
    MORPHO_TRY(validate(p, &s));
    MORPHO_TRY(check_ptr(dweights_f32, "dweights_f32"));
    MORPHO_TRY(check_ptr(dW_phi, "dW_phi"));
    MORPHO_TRY(check_ptr(d_gate_q, "d_gate_q"));
    MORPHO_TRY(check_ptr(d_gate_k, "d_gate_k"));
    MORPHO_TRY(check_ptr(dW_V, "dW_V"));
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    return launch_finalize_weights(s, dweights_f32, alpha, static_cast<__half*>(dW_phi), static_cast<__half*>(dW_V),
                                   static_cast<__half*>(d_gate_q), static_cast<__half*>(d_gate_k),
                                   static_cast<cudaStream_t>(stream));
}

const char* morpho_sm100_last_error(void) { return last_error(); }

int morpho_sm100_last_launch_count(void) { return launch_count(); }

void morpho_sm100_profile_enable(int on) { prof_enable(on != 0); }

void morpho_sm100_profile_select(const char* kernel_name) { prof_select(kernel_name); }

int morpho_sm100_profile_collect(char* names, int name_len, float* total_ms, int* counts, int max_kernels) {
    if (names == nullptr || total_ms == nullptr || counts == nullptr || name_len <= 0 || max_kernels <= 0) return 0;
    return prof_collect(names, name_len, total_ms, counts, max_kernels);
}

int morpho_sm100_device_status(void* stream, int reset, uint32_t* status_out) {
    clear_error();
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t v = 0;
    MORPHO_CUDA_TRY(cudaMemcpyAsync(&v, dev.status, sizeof(v), cudaMemcpyDeviceToHost, st));
    MORPHO_CUDA_TRY(cudaStreamSynchronize(st));
    if (reset) MORPHO_CUDA_TRY(cudaMemsetAsync(dev.status, 0, sizeof(uint32_t), st));
    if (status_out) *status_out = v;
    if (v != 0)
        return set_error(MORPHO_ERR_TIMEOUT, "device status 0x%08x: kernel %u wait site %u timed out", v, v & 0xFFu,
                         (v >> 8) & 0xFFu);
    return MORPHO_OK;
}

}  // extern "C"
