// torch_ops.cpp -- registers the reference's torch op schemas (namespace morphottention)
// on the CUDA dispatch key and forwards them to the C ABI of libmorpho_sm100.so.
//
// Schemas, argument checks and their messages follow the reference host layer
// (packages/morphottention/csrc/cuda/binder.cpp:6-15, csrc/cuda/dispatch.cpp:3-15,
// csrc/cuda/attention/attention.cpp:9-118).  Differences: a device guard (the reference
// has none), workspace from the torch caching allocator on the current stream, no
// zero-fill of the gradient outputs (the kernels overwrite them), and extra ops:
// set_grad_mode / get_grad_mode select full gradients (default) or the reference
// kernel's gradient semantics; set_cube_projection / set_mask_diag (and their getters)
// select the reference's compile-time variants (HardTanh01 / Identity projection, the
// diagonal mask); set_score / get_score / get_score_tau select the soft-morphology
// aggregation (the reference's unused morfology/soft_morph.cuh); get_options returns all of
// them at once.  These process-wide settings apply to the reference-schema ops `forward` and
// `backward` at the moment each is called.  forward_save / backward_saved keep the
// projection of the forward for the backward instead of recomputing it, and take every
// option as an explicit argument, so a backward always runs the variant its forward ran
// (the autograd Functions capture the settings when the forward runs); backward_saved_tau
// also returns dL/dtau of the soft-morphology score (a learnable temperature).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <atomic>
#include <vector>

#include "../../include/morpho_sm100.h"

namespace {

std::atomic<int> g_grad_mode{MORPHO_GRAD_FULL};
std::atomic<int> g_projection{MORPHO_PROJ_SIGMOID};
std::atomic<int> g_mask_diag{0};
std::atomic<int> g_score{MORPHO_SCORE_SOFTMAX};
std::atomic<float> g_tau{1.0f};

void check(const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.scalar_type() == at::kHalf, name, " must be float16");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

// Options of one call: the process-wide settings, or explicit values (forward_save /
// backward_saved).
struct Options {
    int grad_mode, projection, mask_diag, score;
    float tau;
};

Options current_options() {
    return {g_grad_mode.load(), g_projection.load(), g_mask_diag.load(), g_score.load(), g_tau.load()};
}

Options explicit_options(int64_t grad_mode, int64_t projection, int64_t mask_diag, int64_t score, double tau) {
    TORCH_CHECK(grad_mode == MORPHO_GRAD_FULL || grad_mode == MORPHO_GRAD_REFERENCE,
                "grad mode must be 0 (full) or 1 (reference)");
    TORCH_CHECK(projection == MORPHO_PROJ_SIGMOID || projection == MORPHO_PROJ_HARDTANH01 ||
                    projection == MORPHO_PROJ_IDENTITY,
                "cube projection must be 0 (sigmoid), 1 (hardtanh01) or 2 (identity)");
    TORCH_CHECK(mask_diag == 0 || mask_diag == 1, "mask_diag must be 0 or 1");
    TORCH_CHECK(score == MORPHO_SCORE_SOFTMAX || score == MORPHO_SCORE_DILATION || score == MORPHO_SCORE_EROSION,
                "score must be 0 (softmax), 1 (dilation) or 2 (erosion)");
    return {static_cast<int>(grad_mode), static_cast<int>(projection), static_cast<int>(mask_diag),
            static_cast<int>(score), static_cast<float>(tau)};
}

morpho_problem_t problem(const at::Tensor& X, int64_t H, int64_t cube_m, double scale, bool causal,
                         const Options& o) {
    morpho_problem_t p;
    p.B = static_cast<int32_t>(X.size(0));
    p.N = static_cast<int32_t>(X.size(1));
    p.D = static_cast<int32_t>(X.size(2));
    p.H = static_cast<int32_t>(H);
    p.cube_m = static_cast<int32_t>(cube_m);
    p.scale = static_cast<float>(scale);
    p.causal = causal ? 1 : 0;
    p.grad_mode = o.grad_mode;
    p.projection = o.projection;
    p.mask_diag = o.mask_diag;
    p.score = o.score;
    p.tau = o.tau;
    return p;
}

void check_shapes(const at::Tensor& X, const at::Tensor& W_phi, const at::Tensor& gate_q, const at::Tensor& gate_k,
                  const at::Tensor& W_V, int64_t H, int64_t cube_m) {
    TORCH_CHECK(X.dim() == 3, "X must be [B, N, D]");
    const int64_t D = X.size(2);
    TORCH_CHECK(H > 0 && D % H == 0, "D must be divisible by H");
    const int64_t head_dim_v = D / H;
    TORCH_CHECK(W_phi.dim() == 2 && W_phi.size(0) == D && W_phi.size(1) == H * cube_m, "W_phi must be [D, H*cube_m]");
    TORCH_CHECK(W_V.dim() == 2 && W_V.size(0) == D && W_V.size(1) == H * head_dim_v, "W_V must be [D, H*head_dim_v]");
    TORCH_CHECK(gate_q.dim() == 2 && gate_q.size(0) == H && gate_q.size(1) == cube_m, "gate_q must be [H, cube_m]");
    TORCH_CHECK(gate_k.dim() == 2 && gate_k.size(0) == H && gate_k.size(1) == cube_m, "gate_k must be [H, cube_m]");
}

std::vector<at::Tensor> forward_impl(const at::Tensor& X, const at::Tensor& W_phi, const at::Tensor& gate_q,
                                     const at::Tensor& gate_k, const at::Tensor& W_V, int64_t H, int64_t cube_m,
                                     double scale, bool causal, bool save, const Options& opts) {
    check(X, "X");
    check(W_phi, "W_phi");
    check(gate_q, "gate_q");
    check(gate_k, "gate_k");
    check(W_V, "W_V");
    check_shapes(X, W_phi, gate_q, gate_k, W_V, H, cube_m);
    const c10::cuda::CUDAGuard guard(X.device());
    const int64_t B = X.size(0), N = X.size(1);
    auto out = at::empty_like(X);
    auto lse = at::empty({B * H, N}, X.options().dtype(at::kFloat));
    morpho_problem_t p = problem(X, H, cube_m, scale, causal, opts);
    const size_t ws_bytes = save ? morpho_sm100_saved_bytes(&p) : morpho_sm100_forward_workspace_size(&p);
    TORCH_CHECK(ws_bytes > 0, "morphottention forward: unsupported problem: ", morpho_sm100_last_error());
    auto ws = at::empty({static_cast<int64_t>(ws_bytes)}, X.options().dtype(at::kByte));
    auto stream = at::cuda::getCurrentCUDAStream(X.device().index());
    const int rc =
        save ? morpho_sm100_forward_save(&p, X.data_ptr(), W_phi.data_ptr(), gate_q.data_ptr(), gate_k.data_ptr(),
                                         W_V.data_ptr(), out.data_ptr(), lse.data_ptr<float>(), ws.data_ptr(),
                                         ws_bytes, static_cast<void*>(stream.stream()))
             : morpho_sm100_forward(&p, X.data_ptr(), W_phi.data_ptr(), gate_q.data_ptr(), gate_k.data_ptr(),
                                    W_V.data_ptr(), out.data_ptr(), lse.data_ptr<float>(), ws.data_ptr(), ws_bytes,
                                    static_cast<void*>(stream.stream()));
    TORCH_CHECK(rc == MORPHO_OK, "morphottention forward failed (", rc, "): ", morpho_sm100_last_error());
    if (save) return {out, lse, ws};
    return {out, lse};
}

std::vector<at::Tensor> morpho_forward(const at::Tensor& X, const at::Tensor& W_phi, const at::Tensor& gate_q,
                                       const at::Tensor& gate_k, const at::Tensor& W_V, int64_t H, int64_t cube_m,
                                       double scale, bool causal) {
    return forward_impl(X, W_phi, gate_q, gate_k, W_V, H, cube_m, scale, causal, false, current_options());
}

// As forward, with the options given explicitly, plus a third output: the uint8 buffer of
// projection outputs that backward_saved reads.
std::vector<at::Tensor> morpho_forward_save(const at::Tensor& X, const at::Tensor& W_phi, const at::Tensor& gate_q,
                                            const at::Tensor& gate_k, const at::Tensor& W_V, int64_t H,
                                            int64_t cube_m, double scale, bool causal, int64_t projection,
                                            int64_t mask_diag, int64_t score, double tau) {
    return forward_impl(X, W_phi, gate_q, gate_k, W_V, H, cube_m, scale, causal, true,
                        explicit_options(MORPHO_GRAD_FULL, projection, mask_diag, score, tau));
}

std::vector<at::Tensor> backward_impl(const at::Tensor& grad_out, const at::Tensor* saved, const at::Tensor& X,
                                      const at::Tensor& W_phi, const at::Tensor& gate_q, const at::Tensor& gate_k,
                                      const at::Tensor& W_V, const at::Tensor& out, const at::Tensor& lse, int64_t H,
                                      int64_t cube_m, double scale, bool causal, const Options& opts,
                                      bool with_dtau = false) {
    TORCH_CHECK(grad_out.is_cuda() && X.is_cuda(), "Gradient output and X must be a CUDA tensors");
    check(grad_out, "grad_out");
    check(X, "X");
    check(W_phi, "W_phi");
    check(gate_q, "gate_q");
    check(gate_k, "gate_k");
    check(W_V, "W_V");
    check(out, "out");
    TORCH_CHECK(lse.is_cuda(), "lse must be a CUDA tensor");
    TORCH_CHECK(lse.scalar_type() == at::kFloat, "lse must be float32");
    TORCH_CHECK(lse.is_contiguous(), "lse must be contiguous");
    TORCH_CHECK(X.dim() == 3, "X must be [B, N, D]");
    const int64_t B = X.size(0), N = X.size(1), D = X.size(2);
    TORCH_CHECK(H > 0 && D % H == 0, "D must be divisible by H");
    TORCH_CHECK(grad_out.sizes() == X.sizes(), "grad_out must match X shape [B, N, D]");
    TORCH_CHECK(out.sizes() == X.sizes(), "out must match X shape [B, N, D]");
    check_shapes(X, W_phi, gate_q, gate_k, W_V, H, cube_m);
    TORCH_CHECK(lse.dim() == 2 && lse.size(0) == B * H && lse.size(1) == N, "lse must be [B*H, N]");
    const c10::cuda::CUDAGuard guard(X.device());
    auto dX = at::empty_like(X);
    auto dW_phi = at::empty_like(W_phi);
    auto d_gate_q = at::empty_like(gate_q);
    auto d_gate_k = at::empty_like(gate_k);
    auto dW_V = at::empty_like(W_V);
    morpho_problem_t p = problem(X, H, cube_m, scale, causal, opts);
    if (saved != nullptr) {
        TORCH_CHECK(saved->is_cuda() && saved->scalar_type() == at::kByte && saved->is_contiguous(),
                    "saved must be the contiguous uint8 CUDA tensor forward_save returned");
        TORCH_CHECK(static_cast<size_t>(saved->numel()) >= morpho_sm100_saved_bytes(&p),
                    "saved does not match this problem");
    }
    const size_t ws_bytes = saved != nullptr ? morpho_sm100_backward_saved_workspace_size(&p)
                                             : morpho_sm100_backward_workspace_size(&p);
    TORCH_CHECK(ws_bytes > 0, "morphottention backward: unsupported problem: ", morpho_sm100_last_error());
    auto ws = at::empty({static_cast<int64_t>(ws_bytes)}, X.options().dtype(at::kByte));
    auto stream = at::cuda::getCurrentCUDAStream(X.device().index());
    // the temperature gradient exists in the library's fp32 weight-gradient bucket only (its last
    // element); the fp16 weight gradients are then finalized from the bucket
    at::Tensor bucket;
    if (with_dtau) {
        TORCH_CHECK(p.score != MORPHO_SCORE_SOFTMAX, "the temperature gradient needs the dilation or erosion score");
        bucket = at::empty({static_cast<int64_t>(morpho_sm100_weight_grad_elems(&p))}, X.options().dtype(at::kFloat));
    }
    float* dweights = with_dtau ? bucket.data_ptr<float>() : nullptr;
    const int rc =
        saved != nullptr
            ? morpho_sm100_backward_saved(&p, grad_out.data_ptr(), saved->data_ptr(), saved->numel(), X.data_ptr(),
                                          W_phi.data_ptr(), gate_q.data_ptr(), gate_k.data_ptr(), W_V.data_ptr(),
                                          out.data_ptr(), lse.data_ptr<float>(), dX.data_ptr(), dW_phi.data_ptr(),
                                          d_gate_q.data_ptr(), d_gate_k.data_ptr(), dW_V.data_ptr(), dweights,
                                          ws.data_ptr(), ws_bytes, static_cast<void*>(stream.stream()))
            : morpho_sm100_backward(&p, grad_out.data_ptr(), X.data_ptr(), W_phi.data_ptr(), gate_q.data_ptr(),
                                    gate_k.data_ptr(), W_V.data_ptr(), out.data_ptr(), lse.data_ptr<float>(),
                                    dX.data_ptr(), dW_phi.data_ptr(), d_gate_q.data_ptr(), d_gate_k.data_ptr(),
                                    dW_V.data_ptr(), nullptr, ws.data_ptr(), ws_bytes,
                                    static_cast<void*>(stream.stream()));
    TORCH_CHECK(rc == MORPHO_OK, "morphottention backward failed (", rc, "): ", morpho_sm100_last_error());
    if (!with_dtau) return {dX, dW_phi, d_gate_q, d_gate_k, dW_V};
    const int rc2 = morpho_sm100_finalize_weight_grads(&p, bucket.data_ptr<float>(), 1.0f, dW_phi.data_ptr(),
                                                       d_gate_q.data_ptr(), d_gate_k.data_ptr(), dW_V.data_ptr(),
                                                       static_cast<void*>(stream.stream()));
    TORCH_CHECK(rc2 == MORPHO_OK, "morphottention backward failed (", rc2, "): ", morpho_sm100_last_error());
    return {dX, dW_phi, d_gate_q, d_gate_k, dW_V, bucket.narrow(0, bucket.numel() - 1, 1).reshape({})};
}

std::vector<at::Tensor> morpho_backward(const at::Tensor& grad_out, const at::Tensor& X, const at::Tensor& W_phi,
                                        const at::Tensor& gate_q, const at::Tensor& gate_k, const at::Tensor& W_V,
                                        const at::Tensor& out, const at::Tensor& lse, int64_t H, int64_t cube_m,
                                        double scale, bool causal) {
    return backward_impl(grad_out, nullptr, X, W_phi, gate_q, gate_k, W_V, out, lse, H, cube_m, scale, causal,
                         current_options());
}

std::vector<at::Tensor> morpho_backward_saved(const at::Tensor& grad_out, const at::Tensor& saved, const at::Tensor& X,
                                              const at::Tensor& W_phi, const at::Tensor& gate_q,
                                              const at::Tensor& gate_k, const at::Tensor& W_V, const at::Tensor& out,
                                              const at::Tensor& lse, int64_t H, int64_t cube_m, double scale,
                                              bool causal, int64_t grad_mode, int64_t projection, int64_t mask_diag,
                                              int64_t score, double tau) {
    return backward_impl(grad_out, &saved, X, W_phi, gate_q, gate_k, W_V, out, lse, H, cube_m, scale, causal,
                         explicit_options(grad_mode, projection, mask_diag, score, tau));
}

// backward_saved plus dL/dtau of the soft-morphology score as a sixth output (0-dim fp32).
std::vector<at::Tensor> morpho_backward_saved_tau(const at::Tensor& grad_out, const at::Tensor& saved,
                                                  const at::Tensor& X, const at::Tensor& W_phi,
                                                  const at::Tensor& gate_q, const at::Tensor& gate_k,
                                                  const at::Tensor& W_V, const at::Tensor& out, const at::Tensor& lse,
                                                  int64_t H, int64_t cube_m, double scale, bool causal,
                                                  int64_t grad_mode, int64_t projection, int64_t mask_diag,
                                                  int64_t score, double tau) {
    return backward_impl(grad_out, &saved, X, W_phi, gate_q, gate_k, W_V, out, lse, H, cube_m, scale, causal,
                         explicit_options(grad_mode, projection, mask_diag, score, tau), true);
}

int64_t set_grad_mode(int64_t mode) {
    TORCH_CHECK(mode == MORPHO_GRAD_FULL || mode == MORPHO_GRAD_REFERENCE, "grad mode must be 0 (full) or 1 (reference)");
    return g_grad_mode.exchange(static_cast<int>(mode));
}

int64_t get_grad_mode() { return g_grad_mode.load(); }

int64_t set_cube_projection(int64_t proj) {
    TORCH_CHECK(proj == MORPHO_PROJ_SIGMOID || proj == MORPHO_PROJ_HARDTANH01 || proj == MORPHO_PROJ_IDENTITY,
                "cube projection must be 0 (sigmoid), 1 (hardtanh01) or 2 (identity)");
    return g_projection.exchange(static_cast<int>(proj));
}

int64_t get_cube_projection() { return g_projection.load(); }

int64_t set_mask_diag(int64_t on) {
    TORCH_CHECK(on == 0 || on == 1, "mask_diag must be 0 or 1");
    return g_mask_diag.exchange(static_cast<int>(on));
}

int64_t get_mask_diag() { return g_mask_diag.load(); }

int64_t set_score(int64_t score, double tau) {
    TORCH_CHECK(score == MORPHO_SCORE_SOFTMAX || score == MORPHO_SCORE_DILATION || score == MORPHO_SCORE_EROSION,
                "score must be 0 (softmax), 1 (dilation) or 2 (erosion)");
    TORCH_CHECK(score == MORPHO_SCORE_SOFTMAX || (tau > 0.0 && tau < 1e30), "tau must be positive and finite");
    g_tau.store(static_cast<float>(tau));
    return g_score.exchange(static_cast<int>(score));
}

int64_t get_score() { return g_score.load(); }

double get_score_tau() { return static_cast<double>(g_tau.load()); }

// [grad_mode, projection, mask_diag, score, tau]: the settings the next forward would run with.
std::vector<double> get_options() {
    const Options o = current_options();
    return {static_cast<double>(o.grad_mode), static_cast<double>(o.projection), static_cast<double>(o.mask_diag),
            static_cast<double>(o.score), static_cast<double>(o.tau)};
}

}  // namespace

TORCH_LIBRARY(morphottention, m) {
    m.def(
        "forward(Tensor X, Tensor W_phi, Tensor gate_q, Tensor gate_k, Tensor W_V, "
        "int H, int cube_m, float scale, bool causal) -> Tensor[]");
    m.def(
        "backward(Tensor grad_out, Tensor X, Tensor W_phi, Tensor gate_q, Tensor gate_k, "
        "Tensor W_V, Tensor out, Tensor lse, int H, int cube_m, float scale, bool causal) -> Tensor[]");
    m.def(
        "forward_save(Tensor X, Tensor W_phi, Tensor gate_q, Tensor gate_k, Tensor W_V, "
        "int H, int cube_m, float scale, bool causal, int projection, int mask_diag, int score, "
        "float tau) -> Tensor[]");
    m.def(
        "backward_saved(Tensor grad_out, Tensor saved, Tensor X, Tensor W_phi, Tensor gate_q, Tensor gate_k, "
        "Tensor W_V, Tensor out, Tensor lse, int H, int cube_m, float scale, bool causal, int grad_mode, "
        "int projection, int mask_diag, int score, float tau) -> Tensor[]");
    m.def(
        "backward_saved_tau(Tensor grad_out, Tensor saved, Tensor X, Tensor W_phi, Tensor gate_q, Tensor gate_k, "
        "Tensor W_V, Tensor out, Tensor lse, int H, int cube_m, float scale, bool causal, int grad_mode, "
        "int projection, int mask_diag, int score, float tau) -> Tensor[]");
    m.def("set_grad_mode(int mode) -> int", &set_grad_mode);
    m.def("get_grad_mode() -> int", &get_grad_mode);
    m.def("set_cube_projection(int proj) -> int", &set_cube_projection);
    m.def("get_cube_projection() -> int", &get_cube_projection);
    m.def("set_mask_diag(int on) -> int", &set_mask_diag);
    m.def("get_mask_diag() -> int", &get_mask_diag);
    m.def("set_score(int score, float tau) -> int", &set_score);
    m.def("get_score() -> int", &get_score);
    m.def("get_score_tau() -> float", &get_score_tau);
    m.def("get_options() -> float[]", &get_options);
}

TORCH_LIBRARY_IMPL(morphottention, CUDA, m) {
    m.impl("forward", &morpho_forward);
    m.impl("backward", &morpho_backward);
    m.impl("forward_save", &morpho_forward_save);
    m.impl("backward_saved", &morpho_backward_saved);
    m.impl("backward_saved_tau", &morpho_backward_saved_tau);
}
