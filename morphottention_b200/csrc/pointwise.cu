// pointwise.cu -- the memory-bound helpers of the backward:
//   * delta_kernel  : delta = rowsum(dO * O) per head (attention.cu:294-311), written as
//                     the -delta slice of the augmented dP MMA, and L = lse + qb' (the
//                     query bias the forward folded into lse)
//   * dz_kernel     : dZ = dL/dphi * phi (1 - phi) for the shared q/k projection and the
//                     per-block gate-gradient partials (project.cuh:70-85, applied to
//                     both the key and -- in full mode -- the query side)
//   * reduce kernel : deterministic sums of the dW split-K partials and gate partials
//                     (the reference uses fp16 atomics: project.cuh:80-96,
//                     attention.cu:386-390)
//   * finalize      : fp32 weight-gradient bucket -> fp16 outputs (data parallel)
// All accesses are 16-byte vectors along the contiguous dimension.
#include "kernels.h"
#include "sm100.cuh"

namespace morpho {
namespace {

constexpr int kTile = 128;
constexpr int kDzLanes = 2;  // token lanes of a dz block

inline int npad_of(int N) { return (N + kTile - 1) / kTile * kTile; }

// One warp per token row of D = H * hd elements.  Lanes hold 8 consecutive elements;
// a head spans hd/8 lanes.
__global__ void __launch_bounds__(256) delta_kernel(const __half* __restrict__ dO, const __half* __restrict__ O,
                                                    const float* __restrict__ lse, const float* __restrict__ qb,
                                                    float* __restrict__ L, __half* __restrict__ qaug, int T, int N,
                                                    int Npad, int D, int H, int hd) {
    const int lane = threadIdx.x & 31;
    const int warps_total = gridDim.x * (blockDim.x >> 5);
    const int lanes_per_head = hd / 8;
    for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps_total) {
        const int b = t / N;
        const int n = t - b * N;
        const uint4* d4 = reinterpret_cast<const uint4*>(dO + static_cast<size_t>(t) * D);
        const uint4* o4 = reinterpret_cast<const uint4*>(O + static_cast<size_t>(t) * D);
        for (int base = 0; base < D / 8; base += 32) {
            const int chunk = base + lane;  // 8-element chunk index within the row
            float acc = 0.f;
            if (chunk < D / 8) {
                const uint4 a = d4[chunk];
                const uint4 c = o4[chunk];
                const __half2* ah = reinterpret_cast<const __half2*>(&a);
                const __half2* ch = reinterpret_cast<const __half2*>(&c);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 x = __half22float2(ah[i]);
                    const float2 y = __half22float2(ch[i]);
                    acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
                }
            }
            for (int off = 1; off < lanes_per_head; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
            if (chunk < D / 8 && (chunk % lanes_per_head) == 0) {
                const int h = chunk / lanes_per_head;
                const size_t bh = static_cast<size_t>(b) * H + h;
                L[bh * Npad + n] = lse[bh * N + n] + qb[bh * Npad + n];
                const __half one = __float2half_rn(1.0f);
                const __half hi = __float2half_rn(-acc);
                const __half lo = __float2half_rn(-acc - __half2float(hi));
                __half2 ones = __halves2half2(one, one), dl = __halves2half2(hi, lo);
                uint4* qa = reinterpret_cast<uint4*>(qaug + (bh * N + n) * 16);
                qa[0] = make_uint4(*reinterpret_cast<uint32_t*>(&ones), *reinterpret_cast<uint32_t*>(&dl), 0u, 0u);
                qa[1] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
    // zero the padded tail [N, Npad) of every (b, h) row
    const int pad = Npad - N;
    if (pad > 0) {
        const int total = (T / N) * H * pad;
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
            const int bh = i / pad;
            const int n = N + (i - bh * pad);
            L[static_cast<size_t>(bh) * Npad + n] = 0.f;
        }
    }
}

// Block = (column threads) x kDzLanes token lanes.  Column thread x owns the columns
// 4x .. 4x+3 (+4*blockDim.x per loop) of the padded dZ space [0, Hp); token lane y takes
// the tokens t0 + y, t0 + y + kDzLanes, ... of the block's contiguous run, so a warp reads
// kDzLanes consecutive tokens of each head per round.  Writes dcat[:, 0:Hp) and the
// block's gate partials, summed over the token lanes in shared memory in a fixed order
// and stored column-major: gate_part[(g * H*m + col) * gridDim.x + block], g = 0 for
// gate_q, 1 for gate_k, so that the reduction reads each column contiguously.
// dphi/dz from phi alone (reference morfology/cube.cuh:28-45): sigmoid phi (1 - phi);
// hardtanh01 1/2 where 0 < phi < 1 (i.e. -1 < z < 1), else 0; identity 1.
template <int PROJ>
__device__ __forceinline__ float cube_grad(float phi) {
    if (PROJ == kProjSigmoid) return phi * (1.0f - phi);
    if (PROJ == kProjHardTanh01) return (phi > 0.0f && phi < 1.0f) ? 0.5f : 0.0f;
    return 1.0f;
}

template <bool FULL, int PROJ>
__global__ void __launch_bounds__(kDzLanes * 256) dz_kernel(const float* __restrict__ phi, const float* __restrict__ dq,
                                                 const float* __restrict__ dk, const float* __restrict__ dcb,
                                                 const float* __restrict__ dqb,
                                                 const __half* __restrict__ gq, const __half* __restrict__ gk,
                                                 __half* __restrict__ dcat, float* __restrict__ gate_part, int T,
                                                 int N, int Npad, int H, int m, int Hp, int Cp, int tokens_per_block) {
    __shared__ float4 red[kDzLanes - 1][2][256];
    const int Hm = H * m;
    const int tl = threadIdx.y;
    const int t0 = blockIdx.x * tokens_per_block;
    const int t1 = min(T, t0 + tokens_per_block);
    // every thread runs the same number of column rounds (the block synchronises in each)
    for (int base = 0; base < Hp; base += blockDim.x * 4) {
        const int col0 = base + threadIdx.x * 4;
        const bool cols = col0 < Hp;
        const bool live = col0 < Hm;  // m is a multiple of 16, so 4 columns never straddle heads
        const int h = live ? col0 / m : 0;
        const int c = col0 - h * m;
        float g_q[4] = {0.f, 0.f, 0.f, 0.f}, g_k[4] = {0.f, 0.f, 0.f, 0.f};
        float aq[4] = {0.f, 0.f, 0.f, 0.f}, ak[4] = {0.f, 0.f, 0.f, 0.f};
        if (live) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                g_q[i] = __half2float(gq[col0 + i]);
                g_k[i] = __half2float(gk[col0 + i]);
            }
        }
#pragma unroll 4
        for (int t = t0 + tl; cols && t < t1; t += kDzLanes) {
            uint2 out = make_uint2(0u, 0u);
            if (live) {
                const int b = t / N;
                const int n = t - b * N;
                const size_t row = static_cast<size_t>(b) * H + h;
                const size_t off = (row * N + n) * m + c;
                const float4 f = *reinterpret_cast<const float4*>(phi + off);
                const float4 kk = *reinterpret_cast<const float4*>(dk + off);
                const float db = dcb[row * Npad + n];
                const float dqbv = dqb != nullptr ? dqb[row * Npad + n] : 0.f;
                float4 qq = make_float4(0.f, 0.f, 0.f, 0.f);
                if (FULL) qq = *reinterpret_cast<const float4*>(dq + off);
                const float fv[4] = {f.x, f.y, f.z, f.w};
                const float kv[4] = {kk.x, kk.y, kk.z, kk.w};
                const float qv[4] = {qq.x, qq.y, qq.z, qq.w};
                float dz[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    // dk_c = dk + gate_q*dcb (centered query codes), so
                    //   dL/dphi = dq*gq + dk*gk + dcb*gq*gk = dq*gq + dk_c*gk
                    //   d gate_k += dk*phi + dcb*gq*phi = dk_c*phi
                    //   d gate_q += dq*phi + dcb*gk*phi
                    //   d gate_k += dqb*q = dqb*gq*phi  (qbias = sum_c gk q: 0 for the softmax
                    //   score, whose rows are shift-invariant; dq already holds the q path)
                    float dphi = kv[i] * g_k[i];
                    if (FULL) dphi = fmaf(qv[i], g_q[i], dphi);
                    dz[i] = dphi * cube_grad<PROJ>(fv[i]);
                    float gqi = db * g_k[i] * fv[i];
                    if (FULL) gqi = fmaf(qv[i], fv[i], gqi);
                    aq[i] += gqi;
                    ak[i] += (kv[i] + dqbv * g_q[i]) * fv[i];
                }
                out = make_uint2(pack_half2(dz[0], dz[1]), pack_half2(dz[2], dz[3]));
            }
            *reinterpret_cast<uint2*>(dcat + static_cast<size_t>(t) * Cp + col0) = out;
        }
        // token lanes 1.. hand their partials to lane 0, which adds them in lane order
        if (tl > 0) {
            red[tl - 1][0][threadIdx.x] = make_float4(aq[0], aq[1], aq[2], aq[3]);
            red[tl - 1][1][threadIdx.x] = make_float4(ak[0], ak[1], ak[2], ak[3]);
        }
        __syncthreads();
        if (tl == 0 && live) {
#pragma unroll
            for (int y = 0; y < kDzLanes - 1; ++y) {
                const float4 vq = red[y][0][threadIdx.x];
                const float4 vk = red[y][1][threadIdx.x];
                aq[0] += vq.x, aq[1] += vq.y, aq[2] += vq.z, aq[3] += vq.w;
                ak[0] += vk.x, ak[1] += vk.y, ak[2] += vk.z, ak[3] += vk.w;
            }
            const size_t nb = gridDim.x;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                gate_part[static_cast<size_t>(col0 + i) * nb + blockIdx.x] = aq[i];
                gate_part[static_cast<size_t>(Hm + col0 + i) * nb + blockIdx.x] = ak[i];
            }
        }
        __syncthreads();
    }
}

// Sum split partials.  Output index space: [dW_phi D*Hm | dW_V D*D | gq Hm | gk Hm].
// Blocks [0, main_blocks) sum the dW split-K partials, four consecutive outputs per thread
// (rows of Hm or D are multiples of 16 elements); the remaining blocks give each gate
// output one warp, whose lanes take every 32nd dz block and combine by a fixed shuffle
// tree (deterministic).
__global__ void __launch_bounds__(256) reduce_weights_kernel(const float* __restrict__ part, int splits,
                                                             const float* __restrict__ gate_part, int gate_blocks,
                                                             float* __restrict__ bucket, __half* __restrict__ dW_phi,
                                                             __half* __restrict__ dW_V, __half* __restrict__ dgq,
                                                             __half* __restrict__ dgk, int D, int Hm, int Hp, int Cp,
                                                             int main_blocks) {
    const long long n_phi = static_cast<long long>(D) * Hm;
    const long long n_v = static_cast<long long>(D) * D;
    const long long plane = static_cast<long long>(D) * Cp;
    if (static_cast<int>(blockIdx.x) < main_blocks) {
        const long long quads = (n_phi + n_v) / 4;
        for (long long qd = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; qd < quads;
             qd += static_cast<long long>(main_blocks) * blockDim.x) {
            const long long i = qd * 4;
            long long src;
            if (i < n_phi) {
                const long long d = i / Hm;
                src = d * Cp + (i - d * Hm);
            } else {
                const long long k = i - n_phi;
                const long long d = k / D;
                src = d * Cp + Hp + (k - d * D);
            }
            float4 acc = *reinterpret_cast<const float4*>(part + src);
            for (int z = 1; z < splits; ++z) {
                const float4 v = *reinterpret_cast<const float4*>(part + z * plane + src);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            if (bucket != nullptr) {
                *reinterpret_cast<float4*>(bucket + i) = acc;
            } else {
                __half* dst = i < n_phi ? dW_phi + i : dW_V + (i - n_phi);
                *reinterpret_cast<uint2*>(dst) = make_uint2(pack_half2(acc.x, acc.y), pack_half2(acc.z, acc.w));
            }
        }
        return;
    }
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x - main_blocks) * (blockDim.x >> 5);
    for (int k = (blockIdx.x - main_blocks) * (blockDim.x >> 5) + (threadIdx.x >> 5); k < 2 * Hm; k += warps) {
        const int g = k < Hm ? 0 : 1;
        const int col = k - g * Hm;
        // the column's gate_blocks partials are contiguous: lane l sums blocks l, l+32, ...
        // eight loads at a time, then a fixed shuffle tree (deterministic)
        const float* src = gate_part + static_cast<long long>(k) * gate_blocks;
        float acc = 0.f;
        for (int blk0 = 0; blk0 < gate_blocks; blk0 += 32 * 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int blk = blk0 + 32 * u + lane;
                v[u] = blk < gate_blocks ? src[blk] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) acc += v[u];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) {
            const long long i = n_phi + n_v + k;
            if (bucket != nullptr)
                bucket[i] = acc;
            else if (g == 0)
                dgq[col] = __float2half_rn(acc);
            else
                dgk[col] = __float2half_rn(acc);
        }
    }
}

__global__ void __launch_bounds__(256) finalize_kernel(const float* __restrict__ bucket, float alpha,
                                                       __half* __restrict__ dW_phi, __half* __restrict__ dW_V,
                                                       __half* __restrict__ dgq, __half* __restrict__ dgk, int D,
                                                       int Hm) {
    const long long n_phi = static_cast<long long>(D) * Hm;
    const long long n_v = static_cast<long long>(D) * D;
    const long long total = n_phi + n_v + 2LL * Hm;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const __half v = __float2half_rn(alpha * bucket[i]);
        if (i < n_phi)
            dW_phi[i] = v;
        else if (i < n_phi + n_v)
            dW_V[i - n_phi] = v;
        else if (i < n_phi + n_v + Hm)
            dgq[i - n_phi - n_v] = v;
        else
            dgk[i - n_phi - n_v - Hm] = v;
    }
}

int grid_for(long long work, int per_block, int cap) {
    long long g = (work + per_block - 1) / per_block;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return static_cast<int>(g);
}

}  // namespace

int launch_delta(const Shape& s, const __half* dO, const __half* O, const float* lse, const float* qb, float* L,
                 __half* qaug, cudaStream_t stream) {
    const int T = static_cast<int>(s.tokens());
    const int grid = grid_for(T, 8, 148 * 16);
    prof_begin(stream, "delta");
    delta_kernel<<<grid, 256, 0, stream>>>(dO, O, lse, qb, L, qaug, T, s.N, npad_of(s.N), s.D, s.H, s.hd);
    MORPHO_LAUNCH_CHECK("delta");
    return MORPHO_OK;
}

int dz_gate_blocks(const Shape& s) {
    const long long T = s.tokens();
    // ~32 tokens per block (16 per token lane): enough warps and loads in flight to cover
    // HBM latency; the gate partials stay small (blocks x 2 x H*m floats)
    return grid_for(T, 32, 8192);
}

// Threads per dz block: one per 4 columns of [0, Hp), a multiple of 32, at most 256.
int dz_threads(const Shape& s) { return min(256, (s.Hp() / 4 + 31) / 32 * 32); }

int launch_dz(const Shape& s, const float* phi, const float* dq, const float* dk, const float* dcb,
              const float* dqb, const __half* gate_q, const __half* gate_k, __half* dcat, float* gate_part,
              int gate_blocks, cudaStream_t stream) {
    const int T = static_cast<int>(s.tokens());
    const int tpb = (T + gate_blocks - 1) / gate_blocks;
    auto kern = s.grad_mode == MORPHO_GRAD_FULL
                    ? (s.proj == kProjSigmoid      ? dz_kernel<true, kProjSigmoid>
                       : s.proj == kProjHardTanh01 ? dz_kernel<true, kProjHardTanh01>
                                                   : dz_kernel<true, kProjIdentity>)
                    : (s.proj == kProjSigmoid      ? dz_kernel<false, kProjSigmoid>
                       : s.proj == kProjHardTanh01 ? dz_kernel<false, kProjHardTanh01>
                                                   : dz_kernel<false, kProjIdentity>);
    prof_begin(stream, "dz");
    kern<<<gate_blocks, dim3(dz_threads(s), kDzLanes), 0, stream>>>(phi, dq, dk, dcb, dqb, gate_q, gate_k, dcat, gate_part, T, s.N,
                                                    npad_of(s.N), s.H, s.m, s.Hp(), s.Cp(), tpb);
    MORPHO_LAUNCH_CHECK("dz");
    return MORPHO_OK;
}

int launch_reduce_weights(const Shape& s, const float* dw_part, int splits, const float* gate_part, int gate_blocks,
                          float* bucket, __half* dW_phi, __half* dW_V, __half* d_gate_q, __half* d_gate_k,
                          cudaStream_t stream) {
    const long long quads = static_cast<long long>(s.D) * (s.Hm() + s.D) / 4;
    const int main_blocks = grid_for(quads, 256, 148 * 8);
    const int gate_warp_blocks = (2 * s.Hm() + 7) / 8;  // one warp per gate output, 8 warps per block
    prof_begin(stream, "reduce_weights");
    reduce_weights_kernel<<<main_blocks + gate_warp_blocks, 256, 0, stream>>>(
        dw_part, splits, gate_part, gate_blocks, bucket, dW_phi, dW_V, d_gate_q, d_gate_k, s.D, s.Hm(), s.Hp(),
        s.Cp(), main_blocks);
    MORPHO_LAUNCH_CHECK("reduce_weights");
    return MORPHO_OK;
}

int launch_finalize_weights(const Shape& s, const float* bucket, float alpha, __half* dW_phi, __half* dW_V,
                            __half* d_gate_q, __half* d_gate_k, cudaStream_t stream) {
    const long long total = static_cast<long long>(s.D) * (s.Hm() + s.D) + 2LL * s.Hm();
    prof_begin(stream, "finalize_weights");
    finalize_kernel<<<grid_for(total, 256, 148 * 8), 256, 0, stream>>>(bucket, alpha, dW_phi, dW_V, d_gate_q,
                                                                       d_gate_k, s.D, s.Hm());
    MORPHO_LAUNCH_CHECK("finalize_weights");
    return MORPHO_OK;
}

}  // namespace morpho
