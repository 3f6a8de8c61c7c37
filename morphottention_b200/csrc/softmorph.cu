// softmorph.cu -- the soft-morphology score on CUDA cores (sm_100a): the exact kernels.  The
// default path is the split one on the tensor cores (softmorph_tc.cu, softmorph_tc_bwd.cu); these
// kernels are its device-side fallback (they return at once unless its range flag is set) and,
// under the MORPHO_SOFT_MORPH_EXACT environment switch, the whole path.
//
// The reference ships a tropical (max-plus / min-plus) soft aggregation in
// csrc/cuda/morfology/soft_morph.cuh:10-77 that no kernel of it calls.  Here it is a run-time
// score variant of the attention path:
//   out[i, c] = sgn * tau * log sum_j exp(sgn * (S_ij + V_jc) / tau)      (lse_finalize, :59-61)
// with the morphological score S_ij = scale * (2 q_i.k_j - qbias_i - cbias_j) of the softmax
// path and sgn = +1 (soft dilation) or -1 (soft erosion).  It is not a contraction (one
// exponential per (i, j, c) -- hd times the softmax path's), so it runs on CUDA cores:
//   * S_ij from the projected codes, 2 k_j.qc_i - qbias_i (qc centered: k.qc = q.k - cbias/2),
//     in fp32; the row constant -scale*qbias_i leaves the log-sum-exp and is added at the end;
//   * per 64-key tile a max pre-pass on packed half2 (HADD2 + HMNMX2, two channels per
//     instruction) gives the stabiliser -- any value near the true maximum is exact for the
//     log-sum-exp, so fp16 rounding there costs nothing;
//   * the sums in fp32 with ex2 (log2 units throughout: a = sgn*log2(e)/tau * (S + V)).
// The backward recomputes P_ijc = exp(sgn (S_ij + V_jc - out_ic) / tau) (morph_weight, :63-67)
// from the forward's m + log2(l) and produces the same intermediates as the softmax path's
// backward (dq, dk, dcb, dV into dcat) plus dqb = dL/dqbias, which the softmax path does not
// have (its rows are shift-invariant):
//   dS_ij = sum_c dO_ic P_ijc,  dV_jc = sum_i dO_ic P_ijc,
//   dq_i = 2 scale sum_j dS_ij (k_j - gate_k/2),  dk_j = 2 scale sum_i dS_ij qc_i,
//   dcbias_j = -scale sum_i dS_ij,  dqbias_i = -scale sum_j dS_ij.
// Two backward kernels own the two reduction directions (query tiles: dq, dqb; key tiles:
// dV, dk, dcb), so nothing is accumulated with atomics.  tau is a fixed hyper-parameter.
//
// Tiles of 64 queries x 64 keys, 256 threads: thread t owns row t / 4 and the channel quarter
// t % 4 (hd / 4 value channels, m / 4 code channels).
#include <cstdlib>

#include "kernels.h"
#include "sm100.cuh"

namespace morpho {
namespace {

constexpr int kT = 64;          // queries (or keys) per tile
constexpr int kThreads = 256;   // 64 rows x 4 channel quarters
constexpr float kLn2 = 0.6931471805599453f;

struct SmArgs {
    int N, Npad, H, D, Hp, Cp, n_tiles;
    int causal, mask_diag;
    float kf;       // sgn * log2(e) / tau: value term, log2 units
    float kf2;      // kf * 2 * scale: code dot-product term
    float out_mul;  // sgn * tau * ln 2
    float two_scale, neg_scale;
    const __half* qc;  // [BH, N, MC] centered query codes
    const __half* kc;  // [BH, N, MC] key codes
    const __half* kd;  // [BH, N, 2 MC] centered key codes, hi | lo
    const __half* v;   // [BH, N, HD]
    const float* qb;   // [BH, Npad] scale * log2(e) * qbias
    const __half* dO;  // [B, N, D]
    __half* out;       // [B, N, D]
    float* o2;         // [BH, N, HD]: m + log2(l) per (i, c); +inf for a row without keys
    float* dq;         // [BH, N, MC]
    float* dqb;        // [BH, Npad]
    float* sg;         // [BH, Npad]: sum_j S_ij dL/dS_ij (for dL/dtau), or NULL
    float* dk;         // [BH, N, MC]
    float* dcb;        // [BH, Npad]
    __half* dcat;      // [B*N, Cp]: dV at columns Hp + h*HD
    const uint32_t* flag;  // fallback flag of the tensor-core forward (null: run unconditionally)
    int run_if_flag;       // 1: run only when *flag != 0 (the exact fallback); 0: only when *flag == 0
};

// Gate of the kernels that exist twice (exact and factorized): true = nothing to do here.
__device__ __forceinline__ bool gated_out(const SmArgs& a) {
    return a.flag != nullptr && ((*a.flag != 0u) != (a.run_if_flag != 0));
}

__device__ __forceinline__ bool dropped(const SmArgs& a, int i, int j) {
    return i >= a.N || j >= a.N || (a.causal && j > i) || (a.mask_diag && j == i);
}

// Stage a [64 x C] fp16 tile of a [BH, N, ld] tensor (rows r0 .. r0+63, columns c0 .. c0+C) as
// fp32 into smem rows of `stride` floats, times `mul`; rows past N are zero.
template <int C>
__device__ __forceinline__ void stage_rows(float* dst, int stride, const __half* src, int ld, int c0, int r0, int N,
                                           float mul) {
    constexpr int V8 = C / 8;  // 16-byte vectors per row
    for (int e = threadIdx.x; e < kT * V8; e += kThreads) {
        const int r = e / V8, u = e - r * V8;
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (r0 + r < N) {
            const uint4 w = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(r0 + r) * ld + c0 + u * 8);
            const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 t = __half22float2(h[k]);
                f[2 * k] = t.x * mul;
                f[2 * k + 1] = t.y * mul;
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) dst[r * stride + u * 8 + k] = f[k];
    }
}

// S'[r][j] = kf2 * (k_j . qc_r) for the thread's 16 keys j = q4*16 .. +16 (or -inf when the
// pair is masked), written to s_tile[r * 65 + j].  `rows` holds the 64 rows of the row-side
// codes, `cols` the 64 rows of the other side, both [64][MC + 1] fp32.
template <int MC>
__device__ __forceinline__ void score_tile(float* s_tile, const float* rows, const float* cols, int r, int q4,
                                           float kf2, const SmArgs& a, int i0, int j0, bool rows_are_queries) {
    float acc[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) acc[t] = 0.f;
#pragma unroll 4
    for (int c = 0; c < MC; ++c) {
        const float x = rows[r * (MC + 1) + c];
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[t] = fmaf(x, cols[(q4 * 16 + t) * (MC + 1) + c], acc[t]);
    }
#pragma unroll
    for (int t = 0; t < 16; ++t) {
        const int other = q4 * 16 + t;
        const int i = rows_are_queries ? i0 + r : i0 + other;
        const int j = rows_are_queries ? j0 + other : j0 + r;
        s_tile[r * 65 + other] = dropped(a, i, j) ? -INFINITY : kf2 * acc[t];
    }
}

// ---------------- forward ----------------
template <int MC, int HD>
__global__ void __launch_bounds__(kThreads) soft_morph_fwd_kernel(const SmArgs a) {
    // fallback of the tensor-core forward: nothing to do unless it flagged an accumulator
    if (gated_out(a)) return;
    constexpr int CPT = HD / 4;  // value channels per thread
    extern __shared__ float sm[];
    float* sq = sm;                          // [64][MC+1] query codes
    float* sk = sq + kT * (MC + 1);          // [64][MC+1] key codes
    float* sv = sk + kT * (MC + 1);          // [64][HD] kf * V
    __half2* sh = reinterpret_cast<__half2*>(sv + kT * HD);  // [64][HD/2] the same, half2
    float* st = reinterpret_cast<float*>(sh + kT * HD / 2);  // [64][65] scores
    const int qt = blockIdx.x, bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int r = threadIdx.x >> 2, q4 = threadIdx.x & 3;
    const int i0 = qt * kT, i = i0 + r;
    const size_t base = static_cast<size_t>(bh) * a.N;
    stage_rows<MC>(sq, MC + 1, a.qc + base * MC, MC, 0, i0, a.N, 1.0f);
    float m[CPT], l[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        m[c] = -INFINITY;
        l[c] = 0.f;
    }
    const int n_kt = a.causal ? qt + 1 : a.n_tiles;
    for (int kt = 0; kt < n_kt; ++kt) {
        const int j0 = kt * kT;
        __syncthreads();  // the previous tile's smem is no longer read
        stage_rows<MC>(sk, MC + 1, a.kc + base * MC, MC, 0, j0, a.N, 1.0f);
        stage_rows<HD>(sv, HD, a.v + base * HD, HD, 0, j0, a.N, a.kf);
        __syncthreads();
        for (int e = threadIdx.x; e < kT * HD / 2; e += kThreads) sh[e] = __floats2half2_rn(sv[2 * e], sv[2 * e + 1]);
        score_tile<MC>(st, sq, sk, r, q4, a.kf2, a, i0, j0, true);
        __syncthreads();
        const float* srow = st + r * 65;
        // stabiliser: the tile's max of S' + V' per channel, on packed half2
        __half2 mx[CPT / 2];
#pragma unroll
        for (int p = 0; p < CPT / 2; ++p) mx[p] = __float2half2_rn(-INFINITY);
        for (int j = 0; j < kT; ++j) {
            const __half2 s2 = __float2half2_rn(srow[j]);
            const __half2* vh = sh + j * (HD / 2) + q4 * (CPT / 2);
#pragma unroll
            for (int p = 0; p < CPT / 2; ++p) mx[p] = __hmax2(mx[p], __hadd2(s2, vh[p]));
        }
#pragma unroll
        for (int p = 0; p < CPT / 2; ++p) {
            const float2 t = __half22float2(mx[p]);
            const float cand[2] = {t.x, t.y};
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int c = 2 * p + u;
                if (cand[u] > m[c]) {
                    l[c] *= ex2(m[c] - cand[u]);  // 0 while m is -inf (l is 0 then too)
                    m[c] = cand[u];
                }
            }
        }
        float mm[CPT];
#pragma unroll
        for (int c = 0; c < CPT; ++c) mm[c] = m[c] == -INFINITY ? 0.f : m[c];
        for (int j = 0; j < kT; ++j) {
            const float s = srow[j];
            const float4* v4 = reinterpret_cast<const float4*>(sv + j * HD + q4 * CPT);
#pragma unroll
            for (int c4 = 0; c4 < CPT / 4; ++c4) {
                const float4 vv = v4[c4];
                l[4 * c4] += ex2(s + vv.x - mm[4 * c4]);
                l[4 * c4 + 1] += ex2(s + vv.y - mm[4 * c4 + 1]);
                l[4 * c4 + 2] += ex2(s + vv.z - mm[4 * c4 + 2]);
                l[4 * c4 + 3] += ex2(s + vv.w - mm[4 * c4 + 3]);
            }
        }
    }
    if (i < a.N && (a.out != nullptr || a.o2 != nullptr)) {
        const float qb = a.qb[static_cast<size_t>(bh) * a.Npad + i];
        __half* orow = a.out == nullptr ? nullptr : a.out + (static_cast<size_t>(b) * a.N + i) * a.D + h * HD + q4 * CPT;
        float* o2row = a.o2 == nullptr ? nullptr : a.o2 + (base + i) * HD + q4 * CPT;
#pragma unroll
        for (int c = 0; c < CPT; c += 2) {
            const bool e0 = l[c] > 0.f, e1 = l[c + 1] > 0.f;
            const float t0 = e0 ? m[c] + log2f(l[c]) : INFINITY;
            const float t1 = e1 ? m[c + 1] + log2f(l[c + 1]) : INFINITY;
            const float out0 = e0 ? a.out_mul * t0 - kLn2 * qb : 0.f;
            const float out1 = e1 ? a.out_mul * t1 - kLn2 * qb : 0.f;
            if (a.out != nullptr) *reinterpret_cast<uint32_t*>(orow + c) = pack_half2(out0, out1);
            if (o2row != nullptr) {
                o2row[c] = t0;
                o2row[c + 1] = t1;
            }
        }
    }
}

// Stage a [64 x HD] fp32 tile of o2 ([BH, N, HD]); rows past N get +inf (P = 0 there).
template <int HD>
__device__ __forceinline__ void stage_o2(float* dst, const float* src, int r0, int N) {
    constexpr int V4 = HD / 4;
    for (int e = threadIdx.x; e < kT * V4; e += kThreads) {
        const int r = e / V4, u = e - r * V4;
        float4 f = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
        if (r0 + r < N) f = *reinterpret_cast<const float4*>(src + static_cast<size_t>(r0 + r) * HD + u * 4);
        *reinterpret_cast<float4*>(dst + r * HD + u * 4) = f;
    }
}

// ---------------- backward, query side: dq, dqb ----------------
template <int MC, int HD>
__global__ void __launch_bounds__(kThreads) soft_morph_bwd_q_kernel(const SmArgs a) {
    if (gated_out(a)) return;
    constexpr int CPT = HD / 4;   // value channels per thread
    constexpr int MPT = MC / 4;   // code channels per thread
    extern __shared__ float sm[];
    float* sq = sm;                       // [64][MC+1] query codes
    float* sk = sq + kT * (MC + 1);       // [64][MC+1] key codes
    float* skd = sk + kT * (MC + 1);      // [64][MC] centered key codes (hi + lo)
    float* sv = skd + kT * MC;            // [64][HD] kf * V
    float* st = sv + kT * HD;             // [64][65] scores, then dS
    const int qt = blockIdx.x, bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int r = threadIdx.x >> 2, q4 = threadIdx.x & 3;
    const int i0 = qt * kT, i = i0 + r;
    const size_t base = static_cast<size_t>(bh) * a.N;
    stage_rows<MC>(sq, MC + 1, a.qc + base * MC, MC, 0, i0, a.N, 1.0f);
    // this thread's dO and m + log2(l) for its row and channel quarter
    float dOr[CPT], o2r[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        dOr[c] = 0.f;
        o2r[c] = INFINITY;
    }
    if (i < a.N) {
        const __half* g = a.dO + (static_cast<size_t>(b) * a.N + i) * a.D + h * HD + q4 * CPT;
        const float* o = a.o2 + (base + i) * HD + q4 * CPT;
#pragma unroll
        for (int c = 0; c < CPT; c += 2) {
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(g + c));
            dOr[c] = t.x;
            dOr[c + 1] = t.y;
            o2r[c] = o[c];
            o2r[c + 1] = o[c + 1];
        }
    }
    float dq[MPT];
#pragma unroll
    for (int c = 0; c < MPT; ++c) dq[c] = 0.f;
    float dqb = 0.f;
    float sdot = 0.f;  // sum_j s_ij dS_ij with s = kf2 (qc_i . k_j), for the temperature gradient
    const int n_kt = a.causal ? qt + 1 : a.n_tiles;
    for (int kt = 0; kt < n_kt; ++kt) {
        const int j0 = kt * kT;
        __syncthreads();
        stage_rows<MC>(sk, MC + 1, a.kc + base * MC, MC, 0, j0, a.N, 1.0f);
        // centered key codes: hi + lo in fp32
        stage_rows<MC>(skd, MC, a.kd + base * 2 * MC, 2 * MC, 0, j0, a.N, 1.0f);
        __syncthreads();
        {
            constexpr int V8 = MC / 8;
            for (int e = threadIdx.x; e < kT * V8; e += kThreads) {
                const int rr = e / V8, u = e - rr * V8;
                if (j0 + rr < a.N) {
                    const uint4 w = *reinterpret_cast<const uint4*>(a.kd + (base + j0 + rr) * 2 * MC + MC + u * 8);
                    const __half2* hh = reinterpret_cast<const __half2*>(&w);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 t = __half22float2(hh[k]);
                        skd[rr * MC + u * 8 + 2 * k] += t.x;
                        skd[rr * MC + u * 8 + 2 * k + 1] += t.y;
                    }
                }
            }
        }
        stage_rows<HD>(sv, HD, a.v + base * HD, HD, 0, j0, a.N, a.kf);
        __syncthreads();
        score_tile<MC>(st, sq, sk, r, q4, a.kf2, a, i0, j0, true);
        __syncthreads();
        // dS_rj = sum_c dO_rc P_rjc, summed over the four channel quarters by shuffles
        float* srow = st + r * 65;
        float dsv[kT / 4];
        for (int jb = 0; jb < kT; jb += kT / 4) {
#pragma unroll
            for (int t = 0; t < kT / 4; ++t) {
                const int j = jb + t;
                const float s = srow[j];
                const float4* v4 = reinterpret_cast<const float4*>(sv + j * HD + q4 * CPT);
                float part = 0.f;
#pragma unroll
                for (int c4 = 0; c4 < CPT / 4; ++c4) {
                    const float4 vv = v4[c4];
                    part = fmaf(dOr[4 * c4], ex2(s + vv.x - o2r[4 * c4]), part);
                    part = fmaf(dOr[4 * c4 + 1], ex2(s + vv.y - o2r[4 * c4 + 1]), part);
                    part = fmaf(dOr[4 * c4 + 2], ex2(s + vv.z - o2r[4 * c4 + 2]), part);
                    part = fmaf(dOr[4 * c4 + 3], ex2(s + vv.w - o2r[4 * c4 + 3]), part);
                }
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                dsv[t] = part;
                if (s > -INFINITY) sdot = fmaf(s, part, sdot);  // dropped pairs: s = -inf, dS = 0
            }
            __syncwarp();
            // every quarter holds the same sums; quarter t%4 == q4 writes them
#pragma unroll
            for (int t = 0; t < kT / 4; ++t)
                if ((t & 3) == q4) srow[jb + t] = dsv[t];
        }
        __syncthreads();
        for (int j = 0; j < kT; ++j) {
            const float ds = srow[j];
            dqb += ds;
#pragma unroll
            for (int c = 0; c < MPT; ++c) dq[c] = fmaf(ds, skd[j * MC + q4 * MPT + c], dq[c]);
        }
    }
    if (i < a.N) {
        float* dst = a.dq + (base + i) * MC + q4 * MPT;
#pragma unroll
        for (int c = 0; c < MPT; ++c) dst[c] = a.two_scale * dq[c];
        if (q4 == 0) {
            const size_t row = static_cast<size_t>(bh) * a.Npad + i;
            a.dqb[row] = a.neg_scale * dqb;
            // S_ij = 2 scale (qc_i . k_j) - scale qbias_i: 2 scale (qc . k) = s * sgn tau ln 2 (= s
            // * out_mul) and scale qbias = ln 2 * qb
            if (a.sg != nullptr) a.sg[row] = a.out_mul * sdot - kLn2 * a.qb[row] * dqb;
        }
    }
}

// ---------------- backward, key side: dV, dk, dcb ----------------
template <int MC, int HD>
__global__ void __launch_bounds__(kThreads) soft_morph_bwd_k_kernel(const SmArgs a) {
    if (gated_out(a)) return;
    constexpr int CPT = HD / 4;
    constexpr int MPT = MC / 4;
    extern __shared__ float sm[];
    float* sk = sm;                       // [64][MC+1] key codes (this CTA's keys)
    float* sq = sk + kT * (MC + 1);       // [64][MC+1] query codes
    float* sg = sq + kT * (MC + 1);       // [64][HD] dO
    float* so = sg + kT * HD;             // [64][HD] m + log2(l)
    float* st = so + kT * HD;             // [64 keys][65] scores, then dS
    const int kt = blockIdx.x, bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int r = threadIdx.x >> 2, q4 = threadIdx.x & 3;
    const int j0 = kt * kT, j = j0 + r;
    const size_t base = static_cast<size_t>(bh) * a.N;
    stage_rows<MC>(sk, MC + 1, a.kc + base * MC, MC, 0, j0, a.N, 1.0f);
    float vr[CPT];  // kf * V for this key row and channel quarter
#pragma unroll
    for (int c = 0; c < CPT; ++c) vr[c] = 0.f;
    if (j < a.N) {
        const __half* src = a.v + (base + j) * HD + q4 * CPT;
#pragma unroll
        for (int c = 0; c < CPT; c += 2) {
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(src + c));
            vr[c] = a.kf * t.x;
            vr[c + 1] = a.kf * t.y;
        }
    }
    float dv[CPT], dk[MPT], dcb = 0.f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) dv[c] = 0.f;
#pragma unroll
    for (int c = 0; c < MPT; ++c) dk[c] = 0.f;
    const int qt0 = a.causal ? kt : 0;
    for (int qt = qt0; qt < a.n_tiles; ++qt) {
        const int i0 = qt * kT;
        __syncthreads();
        stage_rows<MC>(sq, MC + 1, a.qc + base * MC, MC, 0, i0, a.N, 1.0f);
        stage_rows<HD>(sg, HD, a.dO + static_cast<size_t>(b) * a.N * a.D, a.D, h * HD, i0, a.N, 1.0f);
        stage_o2<HD>(so, a.o2 + base * HD, i0, a.N);
        __syncthreads();
        score_tile<MC>(st, sk, sq, r, q4, a.kf2, a, i0, j0, false);  // st[key r][query]
        __syncthreads();
        float* srow = st + r * 65;
        float dsv[kT / 4];
        for (int ib = 0; ib < kT; ib += kT / 4) {
#pragma unroll
            for (int t = 0; t < kT / 4; ++t) {
                const int ii = ib + t;
                const float s = srow[ii];
                const float4* g4 = reinterpret_cast<const float4*>(sg + ii * HD + q4 * CPT);
                const float4* o4 = reinterpret_cast<const float4*>(so + ii * HD + q4 * CPT);
                float part = 0.f;
#pragma unroll
                for (int c4 = 0; c4 < CPT / 4; ++c4) {
                    const float4 gg = g4[c4], oo = o4[c4];
                    const float p0 = ex2(s + vr[4 * c4] - oo.x), p1 = ex2(s + vr[4 * c4 + 1] - oo.y);
                    const float p2 = ex2(s + vr[4 * c4 + 2] - oo.z), p3 = ex2(s + vr[4 * c4 + 3] - oo.w);
                    dv[4 * c4] = fmaf(gg.x, p0, dv[4 * c4]);
                    dv[4 * c4 + 1] = fmaf(gg.y, p1, dv[4 * c4 + 1]);
                    dv[4 * c4 + 2] = fmaf(gg.z, p2, dv[4 * c4 + 2]);
                    dv[4 * c4 + 3] = fmaf(gg.w, p3, dv[4 * c4 + 3]);
                    part = fmaf(gg.x, p0, fmaf(gg.y, p1, fmaf(gg.z, p2, fmaf(gg.w, p3, part))));
                }
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                dsv[t] = part;
            }
            __syncwarp();
#pragma unroll
            for (int t = 0; t < kT / 4; ++t)
                if ((t & 3) == q4) srow[ib + t] = dsv[t];
        }
        __syncthreads();
        for (int ii = 0; ii < kT; ++ii) {
            const float ds = srow[ii];
            dcb += ds;
#pragma unroll
            for (int c = 0; c < MPT; ++c) dk[c] = fmaf(ds, sq[ii * (MC + 1) + q4 * MPT + c], dk[c]);
        }
    }
    if (j < a.N) {
        __half* dvd = a.dcat + (static_cast<size_t>(b) * a.N + j) * a.Cp + a.Hp + h * HD + q4 * CPT;
#pragma unroll
        for (int c = 0; c < CPT; c += 2) *reinterpret_cast<uint32_t*>(dvd + c) = pack_half2(dv[c], dv[c + 1]);
        float* dkd = a.dk + (base + j) * MC + q4 * MPT;
#pragma unroll
        for (int c = 0; c < MPT; ++c) dkd[c] = a.two_scale * dk[c];
        if (q4 == 0) a.dcb[static_cast<size_t>(bh) * a.Npad + j] = a.neg_scale * dcb;
    }
}

template <int MC, int HD>
size_t fwd_smem() {
    return sizeof(float) * (2 * kT * (MC + 1) + kT * HD + kT * HD / 2 + kT * 65);
}
template <int MC, int HD>
size_t bwd_q_smem() {
    return sizeof(float) * (2 * kT * (MC + 1) + kT * MC + kT * HD + kT * 65);
}
template <int MC, int HD>
size_t bwd_k_smem() {
    return sizeof(float) * (2 * kT * (MC + 1) + 2 * kT * HD + kT * 65);
}

SmArgs make_args(const Shape& s, const ProjOut& p) {
    SmArgs a{};
    a.N = s.N;
    a.Npad = (s.N + 127) / 128 * 128;
    a.H = s.H;
    a.D = s.D;
    a.Hp = s.Hp();
    a.Cp = s.Cp();
    a.n_tiles = (s.N + kT - 1) / kT;
    a.causal = s.causal ? 1 : 0;
    a.mask_diag = s.mask_diag ? 1 : 0;
    const float sgn = s.score == kScoreErosion ? -1.0f : 1.0f;
    a.kf = sgn * kLog2e / s.tau;
    a.kf2 = a.kf * 2.0f * s.scale;
    a.out_mul = sgn * s.tau * kLn2;
    a.two_scale = 2.0f * s.scale;
    a.neg_scale = -s.scale;
    a.qc = p.qc;
    a.kc = p.kc;
    a.kd = p.kdq;
    a.v = p.v;
    a.qb = p.qb;
    return a;
}

template <int MC, int HD>
int run_fwd(const SmArgs& a, int BH, cudaStream_t stream) {
    auto kern = soft_morph_fwd_kernel<MC, HD>;
    const size_t smem = fwd_smem<MC, HD>();
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    prof_begin(stream, "soft_morph_fwd");
    kern<<<dim3(a.n_tiles, BH), kThreads, smem, stream>>>(a);
    MORPHO_LAUNCH_CHECK("soft_morph_fwd");
    return MORPHO_OK;
}

// The exact pair; with a.flag set it is the tensor-core backward's guard (runs only when the
// forward flagged an accumulator).
template <int MC, int HD>
int run_bwd(const SmArgs& a, int BH, cudaStream_t stream) {
    auto kq = soft_morph_bwd_q_kernel<MC, HD>;
    auto kk = soft_morph_bwd_k_kernel<MC, HD>;
    const size_t sq = bwd_q_smem<MC, HD>(), sk = bwd_k_smem<MC, HD>();
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sq)));
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kk, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sk)));
    prof_begin(stream, "soft_morph_bwd_q");
    kq<<<dim3(a.n_tiles, BH), kThreads, sq, stream>>>(a);
    MORPHO_LAUNCH_CHECK("soft_morph_bwd_q");
    prof_begin(stream, "soft_morph_bwd_k");
    kk<<<dim3(a.n_tiles, BH), kThreads, sk, stream>>>(a);
    MORPHO_LAUNCH_CHECK("soft_morph_bwd_k");
    return MORPHO_OK;
}

// (cube_m, head_dim) dispatch
template <template <int, int> class F>
int dispatch(const Shape& s, const SmArgs& a, cudaStream_t st) {
    const int BH = s.B * s.H;
#define MORPHO_SM_CASE(M, HDV) \
    if (s.m == M && s.hd == HDV) return F<M, HDV>::run(a, BH, st);
    MORPHO_SM_CASE(16, 32) MORPHO_SM_CASE(16, 64) MORPHO_SM_CASE(16, 128)
    MORPHO_SM_CASE(32, 32) MORPHO_SM_CASE(32, 64) MORPHO_SM_CASE(32, 128)
    MORPHO_SM_CASE(64, 32) MORPHO_SM_CASE(64, 64) MORPHO_SM_CASE(64, 128)
#undef MORPHO_SM_CASE
    return set_error(MORPHO_ERR_INVALID, "soft-morphology score: cube_m %d, head_dim %d not supported", s.m, s.hd);
}

template <int MC, int HD>
struct Fwd {
    static int run(const SmArgs& a, int BH, cudaStream_t st) { return run_fwd<MC, HD>(a, BH, st); }
};
template <int MC, int HD>
struct Bwd {
    static int run(const SmArgs& a, int BH, cudaStream_t st) { return run_bwd<MC, HD>(a, BH, st); }
};

}  // namespace

bool soft_morph_exact_only() {
    const char* e = std::getenv("MORPHO_SOFT_MORPH_EXACT");
    return e != nullptr && e[0] != '\0' && !(e[0] == '0' && e[1] == '\0');
}

int launch_soft_morph_fwd(const Shape& s, const ProjOut& p, __half* out, float* o2, const uint32_t* only_if,
                          cudaStream_t stream) {
    SmArgs a = make_args(s, p);
    a.out = out;
    a.o2 = o2;
    a.flag = only_if;
    a.run_if_flag = 1;
    return dispatch<Fwd>(s, a, stream);
}

int launch_soft_morph_bwd(const Shape& s, const ProjOut& p, const SmBwdScratch* tcx, uint32_t* status,
                          const __half* dO, const float* o2, float* dq, float* dqb, float* sg, float* dk,
                          float* dcb, __half* dcat, cudaStream_t stream) {
    if (p.kdq == nullptr)
        return set_error(MORPHO_ERR_INVALID, "internal: soft-morphology backward needs the centered key codes");
    SmArgs a = make_args(s, p);
    a.dO = dO;
    a.o2 = const_cast<float*>(o2);
    a.dq = dq;
    a.dqb = dqb;
    a.sg = sg;
    a.dk = dk;
    a.dcb = dcb;
    a.dcat = dcat;
    if (!soft_morph_exact_only()) {
        // the split forward that wrote o2 also wrote m, R and the range flag: the tensor-core pair
        // runs when the flag is clear, the exact pair (below) when it is set
        if (tcx == nullptr)
            return set_error(MORPHO_ERR_INVALID, "internal: soft-morphology backward scratch missing");
        MORPHO_TRY(launch_soft_morph_bwd_tc(s, p, *tcx, dO, o2, dq, dqb, sg, dk, dcb, dcat, status, stream));
        a.flag = p.smflag;
        a.run_if_flag = 1;
    }
    return dispatch<Bwd>(s, a, stream);
}

// ---------------- temperature gradient ----------------
// dL/dtau = (1/tau) [sum_ic dO_ic out_ic - sum_ij S_ij dL/dS_ij - sum_jc V_jc dL/dV_jc]: the
// reference's per-(i, c) term (morfology/soft_morph.cuh:67-77) is dtau_ic = (out_ic - sum_j
// P_ijc (S_ij + V_jc)) / tau with dtau = sum_ic dO_ic dtau_ic, and the sum over j of P (S + V)
// splits into the score and value gradients the backward already forms (dL/dS_ij = sum_c dO_ic
// P_ijc, dL/dV_jc = sum_i dO_ic P_ijc).  The query-side kernels leave sum_j S_ij dL/dS_ij per row
// (sg); the value gradient is dcat's dV.  Two launches, fixed summation order (deterministic).
namespace {

struct DtauArgs {
    int N, Npad, H, D, Cp, Hp, chunks;
    float out_mul;  // sgn * tau * ln 2: out = out_mul * o2 - ln 2 * qb
    const float* o2;
    const float* qb;
    const float* sg;
    const __half* dO;
    const __half* v;
    const __half* dcat;
    float* part;  // [BH * chunks]
};

// Block (bh, 32-row chunk), 8 warps; a warp walks rows, its lanes the head's channels.
template <int HD>
__global__ void __launch_bounds__(256) soft_morph_dtau_partial_kernel(const DtauArgs a) {
    __shared__ float red[8];
    const int bh = blockIdx.x, chunk = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float acc = 0.f;
    for (int rr = warp; rr < 32; rr += 8) {
        const int i = chunk * 32 + rr;
        if (i >= a.N) break;
        const size_t row = static_cast<size_t>(bh) * a.Npad + i;
        const size_t vrow = (static_cast<size_t>(bh) * a.N + i) * HD;
        const size_t tok = static_cast<size_t>(b) * a.N + i;
        const float qbl = kLn2 * a.qb[row];
        float t = 0.f;
#pragma unroll
        for (int c = lane; c < HD; c += 32) {
            const float o = a.o2[vrow + c];
            const float out = o == INFINITY ? 0.f : a.out_mul * o - qbl;  // +inf: a row without keys
            t = fmaf(__half2float(a.dO[tok * a.D + h * HD + c]), out, t);
            t = fmaf(-__half2float(a.v[vrow + c]), __half2float(a.dcat[tok * a.Cp + a.Hp + h * HD + c]), t);
        }
        if (lane == 0) t -= a.sg[row];
        acc += t;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float sum = 0.f;
        for (int w = 0; w < 8; ++w) sum += red[w];
        a.part[static_cast<size_t>(bh) * a.chunks + chunk] = sum;
    }
}

__global__ void __launch_bounds__(256) soft_morph_dtau_final_kernel(const float* part, int n, float inv_tau,
                                                                     float* out) {
    __shared__ float red[256];
    float sum = 0.f;
    for (int k = threadIdx.x; k < n; k += 256) sum += part[k];
    red[threadIdx.x] = sum;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[0] = red[0] * inv_tau;
}

}  // namespace

size_t soft_morph_dtau_parts(const Shape& s) {
    return static_cast<size_t>(s.B) * s.H * ((s.N + 31) / 32);
}

int launch_soft_morph_dtau(const Shape& s, const ProjOut& p, const __half* dO, const float* o2, const float* sg,
                           const __half* dcat, float* part, float* dtau, cudaStream_t stream) {
    if (o2 == nullptr || sg == nullptr || part == nullptr || dtau == nullptr)
        return set_error(MORPHO_ERR_INVALID, "internal: temperature gradient buffers missing");
    DtauArgs a;
    a.N = s.N;
    a.Npad = (s.N + 127) / 128 * 128;
    a.H = s.H;
    a.D = s.D;
    a.Cp = s.Cp();
    a.Hp = s.Hp();
    a.chunks = (s.N + 31) / 32;
    const float sgn = s.score == kScoreErosion ? -1.0f : 1.0f;
    a.out_mul = sgn * s.tau * kLn2;
    a.o2 = o2;
    a.qb = p.qb;
    a.sg = sg;
    a.dO = dO;
    a.v = p.v;
    a.dcat = dcat;
    a.part = part;
    const dim3 grid(s.B * s.H, a.chunks);
    prof_begin(stream, "soft_morph_dtau");
    switch (s.hd) {
        case 32: soft_morph_dtau_partial_kernel<32><<<grid, 256, 0, stream>>>(a); break;
        case 64: soft_morph_dtau_partial_kernel<64><<<grid, 256, 0, stream>>>(a); break;
        case 128: soft_morph_dtau_partial_kernel<128><<<grid, 256, 0, stream>>>(a); break;
        default: return set_error(MORPHO_ERR_INVALID, "head_dim %d not supported", s.hd);
    }
    MORPHO_LAUNCH_CHECK("soft_morph_dtau");
    prof_begin(stream, "soft_morph_dtau_final");
    soft_morph_dtau_final_kernel<<<1, 256, 0, stream>>>(part, static_cast<int>(soft_morph_dtau_parts(s)),
                                                        1.0f / s.tau, dtau);
    MORPHO_LAUNCH_CHECK("soft_morph_dtau_final");
    return MORPHO_OK;
}

}  // namespace morpho
