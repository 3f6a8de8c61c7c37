// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.  extern "C" wrappers around the reference's
// own kernel launchers (packages/morphottention/csrc/cuda/attention/attention.cuh:28-38),
// compiled together with the unmodified reference attention.cu by oracle/build_ref.py,
// so that tests can run the reference CUDA kernels through ctypes without registering a
// second `morphottention` torch op namespace.  Exceptions thrown by the reference's
// TORCH_CHECKs are caught and returned as a status plus message.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <exception>

#include "cuda/attention/attention.cuh"

extern "C" {

int ref_forward(const void* X, const void* W_phi, const void* gate_q, const void* gate_k, const void* W_V, void* out,
                float* lse, int B, int N, int D, int H, int cube_m, int head_dim_v, float scale, void* stream,
                char* err, int err_len) {
    try {
        attention_forward_kernel_launcher(
            static_cast<const __half*>(X), static_cast<const __half*>(W_phi), static_cast<const __half*>(gate_q),
            static_cast<const __half*>(gate_k), static_cast<const __half*>(W_V), static_cast<__half*>(out), lse, B,
            N, D, H, cube_m, head_dim_v, scale, static_cast<cudaStream_t>(stream));
    } catch (const std::exception& e) {
        if (err != nullptr && err_len > 0) snprintf(err, err_len, "%s", e.what());
        return 1;
    }
    return 0;
}

int ref_backward(const void* grad_out, const void* X, const void* W_phi, const void* gate_q, const void* gate_k,
                 const void* W_V, const void* out, const float* lse, void* dX, void* dW_phi, void* d_gate_q,
                 void* d_gate_k, void* dW_V, int B, int N, int D, int H, int cube_m, int head_dim_v, float scale,
                 void* stream, char* err, int err_len) {
    try {
        attention_backward_kernel_launcher(
            static_cast<const __half*>(grad_out), static_cast<const __half*>(X), static_cast<const __half*>(W_phi),
            static_cast<const __half*>(gate_q), static_cast<const __half*>(gate_k), static_cast<const __half*>(W_V),
            static_cast<const __half*>(out), lse, static_cast<__half*>(dX), static_cast<__half*>(dW_phi),
            static_cast<__half*>(d_gate_q), static_cast<__half*>(d_gate_k), static_cast<__half*>(dW_V), B, N, D, H,
            cube_m, head_dim_v, scale, static_cast<cudaStream_t>(stream));
    } catch (const std::exception& e) {
        if (err != nullptr && err_len > 0) snprintf(err, err_len, "%s", e.what());
        return 1;
    }
    return 0;
}

}  // extern "C"
