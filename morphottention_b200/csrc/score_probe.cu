// score_probe.cu -- design probe (no reference counterpart): the morphological score on packed
// half2 CUDA-core math, to measure against the tcgen05 score of the attention kernels.
//
// The score S_ij = qc_i . k_j is a K = cube_m contraction (plus rank-1 bias terms the attention
// kernels fold away), so the attention kernels issue it as tcgen05 MMAs.  This kernel is the
// alternative the design was weighed against: every (query, key) pair's dot product with HFMA2
// (cube_m / 2 packed fp16 multiply-adds, fp16 accumulation as a packed-math kernel would run it),
// the two halves added, and a running row maximum with HMNMX2 -- the "score and max reduction on
// CUDA cores" form.  One thread per query row, its codes in registers; key tiles of 128 rows staged
// in shared memory and read as broadcasts.  Output: the row maxima (fp32).
#include "host_common.h"

namespace morpho {
namespace {

constexpr int kProbeTile = 128;

template <int MC>
__global__ void __launch_bounds__(kProbeTile) score_probe_half2_kernel(const __half* __restrict__ qc,
                                                                        const __half* __restrict__ kc, int N,
                                                                        float* __restrict__ rowmax) {
    constexpr int P = MC / 2;  // half2 pairs per code row
    __shared__ __half2 ks[kProbeTile][P];
    const int bh = blockIdx.y;
    const int i = blockIdx.x * kProbeTile + threadIdx.x;
    const size_t base = static_cast<size_t>(bh) * N;
    __half2 q[P];
#pragma unroll
    for (int c = 0; c < P; ++c)
        q[c] = i < N ? reinterpret_cast<const __half2*>(qc + (base + i) * MC)[c] : __float2half2_rn(0.f);
    __half2 best = __float2half2_rn(-65504.f);
    for (int j0 = 0; j0 < N; j0 += kProbeTile) {
        __syncthreads();
        for (int e = threadIdx.x; e < kProbeTile * P; e += kProbeTile) {
            const int r = e / P, c = e - r * P;
            ks[r][c] = j0 + r < N ? reinterpret_cast<const __half2*>(kc + (base + j0 + r) * MC)[c]
                                  : __float2half2_rn(0.f);
        }
        __syncthreads();
        const int jn = min(kProbeTile, N - j0);  // keys of this tile
#pragma unroll 2
        for (int j = 0; j + 1 < jn; j += 2) {
            __half2 a = __float2half2_rn(0.f), b = __float2half2_rn(0.f);
#pragma unroll
            for (int c = 0; c < P; ++c) {
                a = __hfma2(q[c], ks[j][c], a);
                b = __hfma2(q[c], ks[j + 1][c], b);
            }
            // (a.x + a.y, b.x + b.y): the scores of keys j and j + 1
            best = __hmax2(best, __hadd2(__lows2half2(a, b), __highs2half2(a, b)));
        }
        if (jn & 1) {  // the odd last key
            __half2 a = __float2half2_rn(0.f);
#pragma unroll
            for (int c = 0; c < P; ++c) a = __hfma2(q[c], ks[jn - 1][c], a);
            const __half sa = __hadd(__low2half(a), __high2half(a));
            best = __hmax2(best, __halves2half2(sa, sa));
        }
    }
    if (i < N) rowmax[base + i] = fmaxf(__low2float(best), __high2float(best));
}

}  // namespace
}  // namespace morpho

using namespace morpho;

extern "C" MORPHO_API int morpho_sm100_score_probe_half2(const void* qc, const void* kc, int32_t BH, int32_t N,
                                                          int32_t cube_m, float* rowmax, void* stream_arg) {
    clear_error();
    reset_launch_count();
    if (qc == nullptr || kc == nullptr || rowmax == nullptr)
        return set_error(MORPHO_ERR_INVALID, "score probe: NULL pointer");
    if (BH <= 0 || BH > 65535 || N <= 0)
        return set_error(MORPHO_ERR_INVALID, "score probe: bad sizes BH=%d N=%d", BH, N);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_arg);
    const dim3 grid((N + kProbeTile - 1) / kProbeTile, BH);
    const __half* q = static_cast<const __half*>(qc);
    const __half* k = static_cast<const __half*>(kc);
    prof_begin(stream, "score_probe_half2");
    switch (cube_m) {
        case 16: score_probe_half2_kernel<16><<<grid, kProbeTile, 0, stream>>>(q, k, N, rowmax); break;
        case 32: score_probe_half2_kernel<32><<<grid, kProbeTile, 0, stream>>>(q, k, N, rowmax); break;
        case 64: score_probe_half2_kernel<64><<<grid, kProbeTile, 0, stream>>>(q, k, N, rowmax); break;
        default: return set_error(MORPHO_ERR_INVALID, "score probe: cube_m %d not supported (16, 32, 64)", cube_m);
    }
    MORPHO_LAUNCH_CHECK("score_probe_half2");
    return MORPHO_OK;
}
