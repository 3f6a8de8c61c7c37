// softmorph_tc_bwd.cu -- the soft-morphology backward on the tensor cores (sm_100a).
//
// With the forward's split (softmorph_tc.cu), P_ijc = E_S[i,j] E_V[j,c] F_ic where
// E_S = 2^(x_ij - m_i), E_V = 2^(y_jc - R_c) and F = 2^(m_i + R_c - t_ic) (log2 units, m_i the
// forward's row reference, R_c the column maxima, t the forward's per-(i, c) log-sum-exp).
// With G = dO (.) F the gradients of the aggregation are two products and elementwise scalings,
//   dS_ij = E_S[i,j] (G . E_V^T)_ij,        dV_jc = E_V[j,c] (E_S^T . G)_jc,
// and dS feeds the score's chain as in the exact kernels (softmorph.cu):
//   dq_i = 2 scale sum_j dS_ij kd_j,  dqbias_i = -scale sum_j dS_ij,
//   dk_j = 2 scale sum_i dS_ij qc_i,  dcbias_j = -scale sum_i dS_ij.
// All products run as tcgen05 MMAs: the score recompute in kind::f16 (fp16 codes, as the
// forward), everything else in kind::tf32 with fp32 operands (G, E_V and the codes laid out by
// the pre-pass kernels below, E_S / dS written by the CUDA-core warps to TMEM as fp32 and used
// as the A operand).
//   sm_g_kernel       : G [B*H, N, hd] and G^T [B*H, hd, Npad] (fp32, tf32-rounded, 0 past N)
//   sm_evn_kernel     : E_V [B*H, Npad, hd] (the row-major copy; the forward wrote E_V^T)
//   sm_codes_t_kernel : kd^T and qc^T [B*H, m, Npad] in fp32 (kd = hi + lo)
//   sm_bwd_q_kernel   : per 128-query tile: S = qc . k^T, X = G . E_V^T, dS = E_S X -> dq (MMA,
//                       A = dS from TMEM), dqb (row sums)
//   sm_bwd_k_kernel   : per 128-key tile: S^T = k . qc^T, X^T = E_V . G^T, E_S^T and dS^T written
//                       over S^T and X^T in TMEM, dV += E_S^T . G and dk += dS^T . qc (A from TMEM),
//                       dcb (row sums); dV scaled by E_V in the epilogue
// Every (cube_m, head_dim) of the path: the key side's ring stages hold a whole 128-query tile
// where two of them fit in shared memory and a 64-query half tile otherwise (head dim 128); the
// query side runs a 1- to 3-stage ring.  The kernels return at once when the forward set its range
// flag (the exact kernels then run instead).
#include "kernels.h"
#include "sm100.cuh"

namespace morpho {
namespace {

constexpr int kTile = 128;
constexpr int kThreads = 384;  // warps 0-3: TMA, MMA, 2 idle; 4-11: two exponent warps per TMEM lane quarter
constexpr float kLn2f = 0.6931471805599453f;

inline int npad_of(int N) { return (N + kTile - 1) / kTile * kTile; }

// ---------------- pre-pass ----------------
// Block (bh, ib): rows ib*32 .. +32.  G = dO 2^(m_i + R_c - t_ic) (0 where t = +inf: rows
// without keys), written row-major for i < N and transposed (0 past N).
template <int HD>
__global__ void __launch_bounds__(256) sm_g_kernel(const __half* __restrict__ dO, const float* __restrict__ o2,
                                                   const float* __restrict__ mrow, const float* __restrict__ rv,
                                                   float* __restrict__ g, float* __restrict__ gt, int N, int Npad,
                                                   int H, int D) {
    __shared__ float tile[32][HD + 1];
    __shared__ float sm_m[32];
    __shared__ float sR[HD];
    const int bh = blockIdx.x, i0 = blockIdx.y * 32;
    const int b = bh / H, h = bh - b * H;
    if (threadIdx.x < 32) {
        const int i = i0 + threadIdx.x;
        float m = 0.f;
        if (i < N) m = mrow[static_cast<size_t>(bh) * Npad + i];
        sm_m[threadIdx.x] = m == -INFINITY ? 0.f : m;
    }
    if (threadIdx.x < HD) sR[threadIdx.x] = rv[static_cast<size_t>(bh) * HD + threadIdx.x];
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * HD; e += 256) {
        const int r = e / HD, c = e - r * HD;
        const int i = i0 + r;
        float v = 0.f;
        if (i < N) {
            const float go = __half2float(dO[(static_cast<size_t>(b) * N + i) * D + h * HD + c]);
            const float t = o2[(static_cast<size_t>(bh) * N + i) * HD + c];
            v = __uint_as_float(round_tf32(go * ex2(sm_m[r] + sR[c] - t)));
            g[(static_cast<size_t>(bh) * N + i) * HD + c] = v;
        }
        tile[r][c] = v;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * HD; e += 256) {
        const int c = e / 32, r = e - c * 32;
        gt[(static_cast<size_t>(bh) * HD + c) * Npad + i0 + r] = tile[r][c];
    }
}

// E_V [bh][j][c] = tf32(2^(kf V_jc - R_c)), 0 past N.
template <int HD>
__global__ void __launch_bounds__(256) sm_evn_kernel(const __half* __restrict__ v, const float* __restrict__ rv,
                                                     float* __restrict__ evn, int N, int Npad, float kf) {
    __shared__ float sR[HD];
    const int bh = blockIdx.x, j0 = blockIdx.y * 32;
    if (threadIdx.x < HD) sR[threadIdx.x] = rv[static_cast<size_t>(bh) * HD + threadIdx.x];
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * HD; e += 256) {
        const int r = e / HD, c = e - r * HD;
        const int j = j0 + r;
        float val = 0.f;
        if (j < N) val = ex2(fmaf(__half2float(v[(static_cast<size_t>(bh) * N + j) * HD + c]), kf, -sR[c]));
        evn[(static_cast<size_t>(bh) * Npad + j) * HD + c] = __uint_as_float(round_tf32(val));
    }
}

// dst [bh][c][j] = src row j, column c (HILO: src [.., 2MC] = hi | lo, summed), fp32, 0 past N.
template <int MC, bool HILO>
__global__ void __launch_bounds__(256) sm_codes_t_kernel(const __half* __restrict__ src, float* __restrict__ dst,
                                                         int N, int Npad) {
    __shared__ float tile[32][MC + 1];
    const int bh = blockIdx.x, j0 = blockIdx.y * 32;
    constexpr int LD = HILO ? 2 * MC : MC;
    for (int e = threadIdx.x; e < 32 * MC; e += 256) {
        const int r = e / MC, c = e - r * MC;
        const int j = j0 + r;
        float v = 0.f;
        if (j < N) {
            const __half* row = src + (static_cast<size_t>(bh) * N + j) * LD;
            v = __half2float(row[c]);
            if (HILO) v += __half2float(row[MC + c]);
        }
        tile[r][c] = v;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * MC; e += 256) {
        const int c = e / 32, r = e - c * 32;
        dst[(static_cast<size_t>(bh) * MC + c) * Npad + j0 + r] = __uint_as_float(round_tf32(tile[r][c]));
    }
}

constexpr int align1k(int x) { return (x + 1023) / 1024 * 1024; }

// ---------------- query side: dq, dqb ----------------
template <int MC, int HD>
struct QCfg {
    static constexpr int Q_BYTES = kTile * MC * 2;   // f16 codes
    static constexpr int G_BYTES = HD * kTile * 4;   // HD/32 chunks of [128 rows x 128 B]
    static constexpr int K_BYTES = kTile * MC * 2;
    static constexpr int EV_BYTES = HD * kTile * 4;
    static constexpr int KD_BYTES = 4 * MC * 128;    // four 32-key chunks of [MC rows x 128 B]
    static constexpr int OFF_SK = 0, OFF_SEV = align1k(K_BYTES), OFF_SKD = OFF_SEV + EV_BYTES;
    static constexpr int STAGE = OFF_SKD + KD_BYTES;
    static constexpr int OFF_Q = 0, OFF_G = align1k(Q_BYTES), OFF_STAGE = OFF_G + G_BYTES;
    static constexpr int STAGES = (OFF_STAGE + 3 * STAGE + 3072 <= 220 * 1024)   ? 3
                                  : (OFF_STAGE + 2 * STAGE + 3072 <= 220 * 1024) ? 2
                                                                                 : 1;
    static constexpr int OFF_BAR = OFF_STAGE + STAGES * STAGE;
    static constexpr int SMEM_BYTES = OFF_BAR + 2048 + 1024;  // barriers, TMEM slot, 2 x 128 row sums; alignment
    static constexpr int TX_STAGE = K_BYTES + EV_BYTES + KD_BYTES;
    static constexpr uint32_t TM_S = 0, TM_X = 128, TM_D = 256, TM_DQ = 384;
    static constexpr uint32_t QK_ROW = MC * 2;
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
    static_assert(TM_DQ + MC <= 512, "TMEM");
};

struct QArgs {
    int N, Npad, n_qtiles, mask_diag;
    float kf2, two_scale, neg_scale;
    const float* mrow;
    float* dq;    // [BH, N, MC]
    float* dqb;   // [BH, Npad]
    const float* qb;  // [BH, Npad] scale * log2(e) * qbias
    float* sg;    // [BH, Npad] sum_j S_ij dL/dS_ij (for dL/dtau), or NULL
    const uint32_t* flag;
    uint32_t* status;
};

template <int MC, int HD, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    sm_bwd_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmEV,
                    const __grid_constant__ CUtensorMap tmKD, const QArgs args) {
    if (*args.flag != 0u) return;  // the forward's range check failed: the exact kernels run
    using Cfg = QCfg<MC, HD>;
    constexpr int ST = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    // bars: [0,ST) kv_full, [ST,2ST) kv_empty, 2ST q_full, +1 sx_full, +2 sx_free, +3 d_full, +4 dq_done, +5 drain,
    //       +6 rs_full (the second exponent half's row sums are in shared memory)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ST + 7);
    float* rs_half = reinterpret_cast<float*>(tmem_slot + 2);  // [128]
    float* sd_half = rs_half + kTile;                          // [128]
    volatile uint32_t* abort_flag = tmem_slot + 1;
    const int warp = warp_id();
    const int lane = threadIdx.x & 31;
    const int bh = blockIdx.y;
    const int qt = CAUSAL ? (args.n_qtiles - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
    const int q0 = qt * kTile;
    const int n_kv_all = (args.N + kTile - 1) / kTile;
    const int n_kv = CAUSAL ? min(n_kv_all, qt + 1) : n_kv_all;
    const uint32_t kv_full0 = smem_u32(bars), kv_empty0 = smem_u32(bars + ST);
    const uint32_t q_full = smem_u32(bars + 2 * ST);
    const uint32_t sx_full = q_full + 8, sx_free = q_full + 16, d_full = q_full + 24, dq_done = q_full + 32,
                   drain = q_full + 40, rs_full = q_full + 48;
    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(kv_full0 + 8 * s, 1);
            mbar_init(kv_empty0 + 8 * s, 1);
        }
        mbar_init(q_full, 1);
        mbar_init(sx_full, 1);
        mbar_init(sx_free, 8);
        mbar_init(d_full, 8);
        mbar_init(dq_done, 1);
        mbar_init(drain, 1);
        mbar_init(rs_full, 4);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto stage_base = [&](int s) { return smem_u32(smem + Cfg::OFF_STAGE + s * Cfg::STAGE); };

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES + Cfg::G_BYTES);
            tma_load_3d(smem_u32(smem + Cfg::OFF_Q), &tmQ, q_full, 0, q0, bh);
#pragma unroll
            for (int kb = 0; kb < HD / 32; ++kb)
                tma_load_3d(smem_u32(smem + Cfg::OFF_G) + kb * 16384, &tmG, q_full, 32 * kb, q0, bh);
            int issued = 0;
            for (int j = 0; j < n_kv; ++j) {
                const int s = j % ST;
                if (j >= ST && !mbar_wait(kv_empty0 + 8 * s, ((j / ST) & 1) ^ 1, args.status, K_SOFT_MORPH, 41)) {
                    *abort_flag = 1u;
                    break;
                }
                if (*abort_flag) break;
                const int kv0 = j * kTile;
                const uint32_t fb = kv_full0 + 8 * s, sb = stage_base(s);
                mbar_arrive_expect_tx(fb, Cfg::TX_STAGE);
                tma_load_3d(sb + Cfg::OFF_SK, &tmK, fb, 0, kv0, bh);
#pragma unroll
                for (int kb = 0; kb < HD / 32; ++kb) tma_load_3d(sb + Cfg::OFF_SEV + kb * 16384, &tmEV, fb, 32 * kb, kv0, bh);
#pragma unroll
                for (int kb = 0; kb < 4; ++kb) tma_load_3d(sb + Cfg::OFF_SKD + kb * MC * 128, &tmKD, fb, kv0 + 32 * kb, 0, bh);
                ++issued;
            }
            mbar_wait(q_full, 0, args.status, K_SOFT_MORPH, 42);
            if (*abort_flag) {
                for (int i = max(0, issued - ST); i < issued; ++i)
                    mbar_wait(kv_full0 + 8 * (i % ST), (i / ST) & 1, args.status, K_SOFT_MORPH, 42);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t id_s = make_idesc_f16(128, 128, false, false);
            constexpr uint32_t id_x = make_idesc_tf32(128, 128);
            constexpr uint32_t id_dq = make_idesc_tf32(128, MC);
            constexpr uint32_t qk_sw = swizzle_code_for_row_bytes(Cfg::QK_ROW);
            constexpr uint32_t qk_sbo = 8 * Cfg::QK_ROW;
            const uint32_t sQ = smem_u32(smem + Cfg::OFF_Q), sG = smem_u32(smem + Cfg::OFF_G);
            auto issue_sx = [&](int j) {
                const uint32_t sb = stage_base(j % ST);
#pragma unroll
                for (int ks = 0; ks < MC / 16; ++ks)
                    umma_ss(tmem + Cfg::TM_S, make_sdesc(sQ + ks * 32, 16, qk_sbo, qk_sw),
                            make_sdesc(sb + Cfg::OFF_SK + ks * 32, 16, qk_sbo, qk_sw), id_s, ks > 0 ? 1u : 0u);
#pragma unroll
                for (int kb = 0; kb < HD / 32; ++kb)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ss_tf32(tmem + Cfg::TM_X, make_sdesc(sG + kb * 16384 + ks * 32, 16, 1024, SW_128),
                                     make_sdesc(sb + Cfg::OFF_SEV + kb * 16384 + ks * 32, 16, 1024, SW_128), id_x,
                                     (kb > 0 || ks > 0) ? 1u : 0u);
                umma_commit(sx_full);
            };
            auto issue_dq = [&](int j) {
                const uint32_t sb = stage_base(j % ST);
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ts_tf32(tmem + Cfg::TM_DQ, tmem + Cfg::TM_D + kb * 32 + ks * 8,
                                     make_sdesc(sb + Cfg::OFF_SKD + kb * MC * 128 + ks * 32, 16, 1024, SW_128), id_dq,
                                     (j > 0 || kb > 0 || ks > 0) ? 1u : 0u);
                umma_commit(dq_done);
                umma_commit(kv_empty0 + 8 * (j % ST));
            };
            bool ok = mbar_wait(q_full, 0, args.status, K_SOFT_MORPH, 43) &&
                      mbar_wait(kv_full0, 0, args.status, K_SOFT_MORPH, 44);
            if (ok) {
                tc_fence_after();
                issue_sx(0);
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                const int s1 = (j + 1) % ST;
                if (ST > 1 && j + 1 < n_kv) {  // the next scores as soon as S_j, X_j are read
                    if (!mbar_wait(sx_free, j & 1, args.status, K_SOFT_MORPH, 45) ||
                        !mbar_wait(kv_full0 + 8 * s1, ((j + 1) / ST) & 1, args.status, K_SOFT_MORPH, 46)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_sx(j + 1);
                }
                if (!mbar_wait(d_full, j & 1, args.status, K_SOFT_MORPH, 47)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                issue_dq(j);
                if (ST == 1 && j + 1 < n_kv) {  // one stage: the next tile's loads wait for dQ_j
                    if (!mbar_wait(kv_full0, (j + 1) & 1, args.status, K_SOFT_MORPH, 46)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_sx(j + 1);
                }
            }
            if (!ok) {
                *abort_flag = 1u;
                umma_commit(drain);
                mbar_wait(drain, 0, args.status, K_SOFT_MORPH, 48);
            }
        }
    } else if (warp >= 4) {
        const int quad = warp & 3;
        const int half = (warp - 4) >> 2;  // this warp's 64 key columns
        const int r = quad * 32 + lane;
        const int q = q0 + r;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
        float m_r = 0.f;
        if (q < args.N) {
            const float mm = args.mrow[static_cast<size_t>(bh) * args.Npad + q];
            m_r = mm == -INFINITY ? 0.f : mm;
        }
        const float kf2 = args.kf2;
        float rowsum = 0.f;
        float sdot = 0.f;  // sum_j (qc_i . k_j) dS_ij, for the temperature gradient
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int kv0 = j * kTile;
            if (!mbar_wait_warp(sx_full, j & 1, args.status, K_SOFT_MORPH, 49)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const bool need_mask = (kv0 + kTile > args.N) || ((CAUSAL || args.mask_diag) && j == qt);
            uint32_t d[kTile / 2];
#pragma unroll
            for (int c = 0; c < kTile / 2; c += 32) {
                uint32_t sv[32], xv[32];
                tmem_ld32(lane_base + Cfg::TM_S + c, sv);
                tmem_ld32(lane_base + Cfg::TM_X + c, xv);
                tmem_ld_wait();
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    float e = ex2(fmaf(u2f(sv[k]), kf2, -m_r));
                    if (need_mask) {
                        const int kv = kv0 + half * 64 + c + k;
                        if (kv >= args.N || (CAUSAL && kv > q) || (args.mask_diag && kv == q)) e = 0.f;
                    }
                    const float dd = e * u2f(xv[k]);
                    rowsum += dd;
                    sdot = fmaf(u2f(sv[k]), dd, sdot);
                    d[c + k] = __float_as_uint(dd);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sx_free);
            if (j > 0) {  // dQ_{j-1} still reads the D columns
                if (!mbar_wait_warp(dq_done, (j - 1) & 1, args.status, K_SOFT_MORPH, 50)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
#pragma unroll
            for (int c = 0; c < kTile / 2; c += 16) tmem_st16(lane_base + Cfg::TM_D + c, d + c);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_full);
        }
        // the second half hands its row sums to the first, which writes the outputs
        if (half == 1) {
            rs_half[r] = rowsum;
            sd_half[r] = sdot;
            __syncwarp();
            if (lane == 0) mbar_arrive(rs_full);
        } else if (ok && n_kv > 0 && mbar_wait_warp(dq_done, (n_kv - 1) & 1, args.status, K_SOFT_MORPH, 51) &&
                   mbar_wait_warp(rs_full, 0, args.status, K_SOFT_MORPH, 52)) {
            tc_fence_after();
            rowsum += rs_half[r];
            sdot += sd_half[r];
            const uint32_t acc_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll
            for (int c = 0; c < MC; c += 16) {
                uint32_t rr[16];
                tmem_ld16(acc_base + Cfg::TM_DQ + c, rr);
                tmem_ld_wait();
                if (q < args.N) {
                    float4* dst = reinterpret_cast<float4*>(args.dq + (static_cast<size_t>(bh) * args.N + q) * MC + c);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_float4(args.two_scale * u2f(rr[4 * i]), args.two_scale * u2f(rr[4 * i + 1]),
                                             args.two_scale * u2f(rr[4 * i + 2]), args.two_scale * u2f(rr[4 * i + 3]));
                }
            }
            if (q < args.N) {
                const size_t row = static_cast<size_t>(bh) * args.Npad + q;
                args.dqb[row] = args.neg_scale * rowsum;
                // S_ij = 2 scale (qc_i . k_j) - scale qbias_i, and scale qbias = ln 2 * qb
                if (args.sg != nullptr) args.sg[row] = args.two_scale * sdot - kLn2f * args.qb[row] * rowsum;
            }
        } else if (!ok) {
            *abort_flag = 1u;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------- key side: dV, dk, dcb ----------------
template <int MC, int HD>
struct KCfg {
    static constexpr int K_BYTES = kTile * MC * 2;
    static constexpr int EV_BYTES = HD * kTile * 4;
    static constexpr int OFF_K = 0, OFF_EV = align1k(K_BYTES), OFF_STAGE = OFF_EV + EV_BYTES;
    // one ring stage holds QS queries: Qc [QS x MC] f16, G in HD/32 chunks of [QS rows x 128 B],
    // G^T and Qc^T in QS/32 chunks of [HD or MC rows x 128 B]
    static constexpr int stage_bytes(int qs) {
        return align1k(qs * MC * 2) + HD * qs * 4 + (qs / 32) * HD * 128 + (qs / 32) * MC * 128;
    }
    // a whole 128-query tile per stage where two such stages fit, else one 64-query half tile
    static constexpr int QS = (OFF_STAGE + 2 * stage_bytes(128) + 3072 <= 220 * 1024) ? 128 : 64;
    static constexpr int UPS = QS / 64;  // 64-query units per stage
    static constexpr int QC_BYTES = QS * MC * 2;
    static constexpr int G_CHUNK = QS * 128;
    static constexpr int G_BYTES = HD * QS * 4;
    static constexpr int GT_BYTES = (QS / 32) * HD * 128;
    static constexpr int QT_BYTES = (QS / 32) * MC * 128;
    static constexpr int OFF_SQC = 0, OFF_SG = align1k(QC_BYTES), OFF_SGT = OFF_SG + G_BYTES,
                         OFF_SQT = OFF_SGT + GT_BYTES;
    static constexpr int STAGE = OFF_SQT + QT_BYTES;
    static constexpr int STAGES = (OFF_STAGE + 2 * STAGE + 3072 <= 220 * 1024) ? 2 : 1;
    static constexpr int OFF_BAR = OFF_STAGE + STAGES * STAGE;
    static constexpr int SMEM_BYTES = OFF_BAR + 1024 + 1024;  // barriers, TMEM slot, 128 row sums; alignment
    static constexpr int TX_STAGE = QC_BYTES + G_BYTES + GT_BYTES + QT_BYTES;
    static constexpr uint32_t TM_DV = 256, TM_DK = 256 + HD;  // [0, 256): two slots of S^T | X^T halves
    static constexpr uint32_t QK_ROW = MC * 2;
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
    static_assert(TM_DK + MC <= 512, "TMEM");
};

struct KArgs {
    int N, Npad, H, D, Hp, Cp, n_tiles, mask_diag;
    float kf2, two_scale, neg_scale;
    const float* mrow;
    __half* dcat;  // [B*N, Cp]: dV at columns Hp + h*HD
    float* dk;     // [BH, N, MC]
    float* dcb;    // [BH, Npad]
    const uint32_t* flag;
    uint32_t* status;
};

template <int MC, int HD, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    sm_bwd_k_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmEV, const __grid_constant__ CUtensorMap tmG,
                    const __grid_constant__ CUtensorMap tmGT, const __grid_constant__ CUtensorMap tmQT,
                    const KArgs args) {
    if (*args.flag != 0u) return;
    using Cfg = KCfg<MC, HD>;
    constexpr int ST = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    // bars: [0,ST) st_full, [ST,2ST) st_empty, 2ST k_full, +1/+2 sx_full of TMEM slot 0/1, +3/+4 ed_full
    //       of slot 0/1, +5 mm_done, +6 drain, +7 rs_full (the second exponent half's row sums are in
    //       shared memory)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ST + 8);
    float* rs_half = reinterpret_cast<float*>(tmem_slot + 2);  // [128]
    volatile uint32_t* abort_flag = tmem_slot + 1;
    const int warp = warp_id();
    const int lane = threadIdx.x & 31;
    const int kt = blockIdx.x, bh = blockIdx.y;
    const int j0 = kt * kTile;
    const int it0 = CAUSAL ? kt : 0;
    const int n_it = args.n_tiles - it0;
    const uint32_t st_full0 = smem_u32(bars), st_empty0 = smem_u32(bars + ST);
    const uint32_t k_full = smem_u32(bars + 2 * ST);
    const uint32_t sx_full0 = k_full + 8, sx_full1 = k_full + 16, ed_full0 = k_full + 24, ed_full1 = k_full + 32,
                   mm_done = k_full + 40, drain = k_full + 48, rs_full = k_full + 56;
    const int n_u = 2 * n_it;  // 64-query half tiles, alternating between two TMEM slots
    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(st_full0 + 8 * s, 1);
            mbar_init(st_empty0 + 8 * s, 1);
        }
        mbar_init(k_full, 1);
        mbar_init(sx_full0, 1);
        mbar_init(sx_full1, 1);
        mbar_init(ed_full0, 8);
        mbar_init(ed_full1, 8);
        mbar_init(mm_done, 1);
        mbar_init(drain, 1);
        mbar_init(rs_full, 4);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto stage_base = [&](int s) { return smem_u32(smem + Cfg::OFF_STAGE + s * Cfg::STAGE); };

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(k_full, Cfg::K_BYTES + Cfg::EV_BYTES);
            tma_load_3d(smem_u32(smem + Cfg::OFF_K), &tmK, k_full, 0, j0, bh);
#pragma unroll
            for (int kb = 0; kb < HD / 32; ++kb)
                tma_load_3d(smem_u32(smem + Cfg::OFF_EV) + kb * 16384, &tmEV, k_full, 32 * kb, j0, bh);
            int issued = 0;
            const int n_st = n_u / Cfg::UPS;  // ring fills
            for (int i = 0; i < n_st; ++i) {
                const int s = i % ST;
                if (i >= ST && !mbar_wait(st_empty0 + 8 * s, ((i / ST) & 1) ^ 1, args.status, K_SOFT_MORPH, 61)) {
                    *abort_flag = 1u;
                    break;
                }
                if (*abort_flag) break;
                const int q0 = it0 * kTile + i * Cfg::QS;
                const uint32_t fb = st_full0 + 8 * s, sb = stage_base(s);
                mbar_arrive_expect_tx(fb, Cfg::TX_STAGE);
                tma_load_3d(sb + Cfg::OFF_SQC, &tmQ, fb, 0, q0, bh);
#pragma unroll
                for (int kb = 0; kb < HD / 32; ++kb)
                    tma_load_3d(sb + Cfg::OFF_SG + kb * Cfg::G_CHUNK, &tmG, fb, 32 * kb, q0, bh);
#pragma unroll
                for (int c = 0; c < Cfg::QS / 32; ++c) {
                    tma_load_3d(sb + Cfg::OFF_SGT + c * HD * 128, &tmGT, fb, q0 + 32 * c, 0, bh);
                    tma_load_3d(sb + Cfg::OFF_SQT + c * MC * 128, &tmQT, fb, q0 + 32 * c, 0, bh);
                }
                ++issued;
            }
            mbar_wait(k_full, 0, args.status, K_SOFT_MORPH, 62);
            if (*abort_flag) {
                for (int i = max(0, issued - ST); i < issued; ++i)
                    mbar_wait(st_full0 + 8 * (i % ST), (i / ST) & 1, args.status, K_SOFT_MORPH, 62);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // Half tile u (queries (u/2)*128 + (u%2)*64 .. +64) uses TMEM slot u%2: S^T in its columns
            // [0, 64), X^T in [64, 128); the warps write E_S^T and dS^T over them, which dV and dk
            // read.  While the warps work on one slot the tensor pipe runs the other slot's dV / dk
            // and the next half tile's S^T / X^T (issued after those in the same thread, so in order).
            constexpr uint32_t id_s = make_idesc_f16(128, 64, false, false);
            constexpr uint32_t id_x = make_idesc_tf32(128, 64);
            constexpr uint32_t id_dv = make_idesc_tf32(128, HD);
            constexpr uint32_t id_dk = make_idesc_tf32(128, MC);
            constexpr uint32_t qk_sw = swizzle_code_for_row_bytes(Cfg::QK_ROW);
            constexpr uint32_t qk_sbo = 8 * Cfg::QK_ROW;
            const uint32_t sK = smem_u32(smem + Cfg::OFF_K), sEV = smem_u32(smem + Cfg::OFF_EV);
            auto issue_sx = [&](int u) -> bool {
                const int i = u / Cfg::UPS, h = u % Cfg::UPS, s = i % ST;  // ring fill, unit within it
                const uint32_t sb = stage_base(s);
                if (h == 0) {
                    if (!mbar_wait(st_full0 + 8 * s, (i / ST) & 1, args.status, K_SOFT_MORPH, 64)) return false;
                    tc_fence_after();
                }
                const uint32_t dst = tmem + (u & 1) * 128;
#pragma unroll
                for (int ks = 0; ks < MC / 16; ++ks)
                    umma_ss(dst, make_sdesc(sK + ks * 32, 16, qk_sbo, qk_sw),
                            make_sdesc(sb + Cfg::OFF_SQC + h * 64 * Cfg::QK_ROW + ks * 32, 16, qk_sbo, qk_sw), id_s,
                            ks > 0 ? 1u : 0u);
#pragma unroll
                for (int kb = 0; kb < HD / 32; ++kb)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ss_tf32(dst + 64, make_sdesc(sEV + kb * 16384 + ks * 32, 16, 1024, SW_128),
                                     make_sdesc(sb + Cfg::OFF_SG + kb * Cfg::G_CHUNK + h * 8192 + ks * 32, 16, 1024,
                                                SW_128),
                                     id_x, (kb > 0 || ks > 0) ? 1u : 0u);
                umma_commit((u & 1) ? sx_full1 : sx_full0);
                return true;
            };
            // S^T / X^T of unit v go out once its slot's previous reader dV / dk(v - 2) has been
            // issued and its ring fill has been loaded, which needs the fill ST earlier released
            // (its last unit's dV / dk issued): v <= u + 2 and (v/UPS - ST + 1) * UPS - 1 <= u
            int next_sx = 0;
            auto issue_ready = [&](int u) -> bool {
                while (next_sx < n_u && next_sx <= u + 2 &&
                       (next_sx / Cfg::UPS - ST + 1) * Cfg::UPS - 1 <= u) {
                    if (!issue_sx(next_sx)) return false;
                    ++next_sx;
                }
                return true;
            };
            bool ok = mbar_wait(k_full, 0, args.status, K_SOFT_MORPH, 63) && issue_ready(-1);
            for (int u = 0; ok && u < n_u; ++u) {
                const int i = u / Cfg::UPS, h = u % Cfg::UPS, s = i % ST, b = u & 1;
                const uint32_t sb = stage_base(s);
                if (!mbar_wait(b ? ed_full1 : ed_full0, (u >> 1) & 1, args.status, K_SOFT_MORPH, 65)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t src = tmem + b * 128;
#pragma unroll
                for (int c = 0; c < 2; ++c) {  // the unit's two 32-query chunks of the ring fill
                    const int kb = 2 * h + c;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint32_t acc = (u > 0 || c > 0 || ks > 0) ? 1u : 0u;
                        umma_ts_tf32(tmem + Cfg::TM_DV, src + c * 32 + ks * 8,
                                     make_sdesc(sb + Cfg::OFF_SGT + kb * HD * 128 + ks * 32, 16, 1024, SW_128), id_dv,
                                     acc);
                        umma_ts_tf32(tmem + Cfg::TM_DK, src + 64 + c * 32 + ks * 8,
                                     make_sdesc(sb + Cfg::OFF_SQT + kb * MC * 128 + ks * 32, 16, 1024, SW_128), id_dk,
                                     acc);
                    }
                }
                if (h == Cfg::UPS - 1) umma_commit(st_empty0 + 8 * s);
                if (!issue_ready(u)) {
                    ok = false;
                    break;
                }
            }
            if (ok) {
                umma_commit(mm_done);
            } else {
                *abort_flag = 1u;
                umma_commit(drain);
                mbar_wait(drain, 0, args.status, K_SOFT_MORPH, 66);
                umma_commit(mm_done);  // release the epilogue wait
            }
        }
    } else if (warp >= 4) {
        const int quad = warp & 3;
        const int half = (warp - 4) >> 2;  // this warp's 32 of each half tile's 64 query columns
        const int r = quad * 32 + lane;
        const int j = j0 + r;
        const uint32_t row_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
        const float kf2 = args.kf2;
        const float* mrow = args.mrow + static_cast<size_t>(bh) * args.Npad;
        float rowsum = 0.f;
        bool ok = true;
        for (int u = 0; u < n_u; ++u) {
            const int i = u >> 1, h = u & 1, b = u & 1;
            const int q0 = (it0 + i) * kTile;
            const int qc = q0 + h * 64 + half * 32;  // first query of this warp's 32 columns
            if (!mbar_wait_warp(b ? sx_full1 : sx_full0, (u >> 1) & 1, args.status, K_SOFT_MORPH, 67)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const bool need_mask = (j0 + kTile > args.N) || (qc + 32 > args.N) ||
                                   ((CAUSAL || args.mask_diag) && q0 == j0);
            const uint32_t sl = row_base + b * 128 + half * 32;
            uint32_t sv[32], xv[32];
            tmem_ld32(sl, sv);
            tmem_ld32(sl + 64, xv);
            float mv = 0.f;
            if (qc + lane < args.N) {
                const float mm = mrow[qc + lane];
                mv = mm == -INFINITY ? 0.f : mm;
            }
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                const float mq = __shfl_sync(0xffffffffu, mv, k);
                float e = ex2(fmaf(u2f(sv[k]), kf2, -mq));
                if (need_mask) {
                    const int qq = qc + k;
                    if (j >= args.N || qq >= args.N || (CAUSAL && j > qq) || (args.mask_diag && j == qq)) e = 0.f;
                }
                const float dd = e * u2f(xv[k]);
                rowsum += dd;
                sv[k] = __float_as_uint(e);
                xv[k] = __float_as_uint(dd);
            }
            tmem_st16(sl, sv);
            tmem_st16(sl + 16, sv + 16);
            tmem_st16(sl + 64, xv);
            tmem_st16(sl + 80, xv + 16);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(b ? ed_full1 : ed_full0);
        }
        // epilogue by the first half: dV = E_V (.) acc -> dcat, dk, dcb (E_V from the shared-memory
        // tile: wait for it; the second half's row sums from shared memory)
        if (half == 1) {
            rs_half[r] = rowsum;
            __syncwarp();
            if (lane == 0) mbar_arrive(rs_full);
        } else if (ok && mbar_wait_warp(mm_done, 0, args.status, K_SOFT_MORPH, 68) &&
                   mbar_wait_warp(k_full, 0, args.status, K_SOFT_MORPH, 69) &&
                   mbar_wait_warp(rs_full, 0, args.status, K_SOFT_MORPH, 70) && !*abort_flag) {
            tc_fence_after();
            rowsum += rs_half[r];
            const uint32_t acc_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
            const int b = bh / args.H;
            const int h = bh - b * args.H;
            const uint8_t* ev_tile = smem + Cfg::OFF_EV;
#pragma unroll
            for (int c = 0; c < HD; c += 16) {
                uint32_t rr[16];
                tmem_ld16(acc_base + Cfg::TM_DV + c, rr);
                tmem_ld_wait();
                uint32_t pk[8];
#pragma unroll
                for (int u = 0; u < 16; u += 2) {
                    float ev[2];
#pragma unroll
                    for (int w = 0; w < 2; ++w) {
                        const int cc = c + u + w;
                        const int off = (cc >> 5) * 16384 + r * 128 + ((((cc & 31) >> 2) ^ (r & 7)) << 4) + ((cc & 3) << 2);
                        ev[w] = *reinterpret_cast<const float*>(ev_tile + off);
                    }
                    pk[u / 2] = pack_half2(ev[0] * u2f(rr[u]), ev[1] * u2f(rr[u + 1]));
                }
                if (j < args.N) {
                    uint4* dst = reinterpret_cast<uint4*>(args.dcat + (static_cast<size_t>(b) * args.N + j) * args.Cp +
                                                          args.Hp + h * HD + c);
                    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
            }
#pragma unroll
            for (int c = 0; c < MC; c += 16) {
                uint32_t rr[16];
                tmem_ld16(acc_base + Cfg::TM_DK + c, rr);
                tmem_ld_wait();
                if (j < args.N) {
                    float4* dst = reinterpret_cast<float4*>(args.dk + (static_cast<size_t>(bh) * args.N + j) * MC + c);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4)
                        dst[q4] = make_float4(args.two_scale * u2f(rr[4 * q4]), args.two_scale * u2f(rr[4 * q4 + 1]),
                                              args.two_scale * u2f(rr[4 * q4 + 2]), args.two_scale * u2f(rr[4 * q4 + 3]));
                }
            }
            if (j < args.N) args.dcb[static_cast<size_t>(bh) * args.Npad + j] = args.neg_scale * rowsum;
        } else if (!ok) {
            *abort_flag = 1u;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

int tmap_f32_3d(CUtensorMap* map, const float* base, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t box0,
                uint32_t box1) {
    const uint64_t dims[3] = {d0, d1, d2};
    const uint64_t strides[2] = {d0 * 4, d0 * d1 * 4};
    const uint32_t box[3] = {box0, box1, 1};
    return make_tmap(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int MC, int HD, bool CAUSAL>
int run_tc_bwd(const Shape& s, const ProjOut& p, const SmBwdScratch& x, const __half* dO, const float* o2,
               float* dq, float* dqb, float* sg, float* dk, float* dcb, __half* dcat, uint32_t* status,
               cudaStream_t stream) {
    const int BH = s.B * s.H;
    const int N = s.N, Npad = npad_of(N), n_tiles = Npad / kTile;
    const float sgn = s.score == kScoreErosion ? -1.0f : 1.0f;
    const float kf = sgn * 1.4426950408889634f / s.tau;
    const dim3 pre(BH, Npad / 32);
    prof_begin(stream, "soft_morph_tc_g");
    sm_g_kernel<HD><<<pre, 256, 0, stream>>>(dO, o2, p.mrow, p.rv, x.g, x.gt, N, Npad, s.H, s.D);
    MORPHO_LAUNCH_CHECK("soft_morph_tc_g");
    prof_begin(stream, "soft_morph_tc_ev");
    sm_evn_kernel<HD><<<pre, 256, 0, stream>>>(p.v, p.rv, x.evn, N, Npad, kf);
    MORPHO_LAUNCH_CHECK("soft_morph_tc_ev");
    prof_begin(stream, "soft_morph_tc_kd");
    sm_codes_t_kernel<MC, true><<<pre, 256, 0, stream>>>(p.kdq, x.kdt, N, Npad);
    MORPHO_LAUNCH_CHECK("soft_morph_tc_kd");
    prof_begin(stream, "soft_morph_tc_qc");
    sm_codes_t_kernel<MC, false><<<pre, 256, 0, stream>>>(p.qc, x.qct, N, Npad);
    MORPHO_LAUNCH_CHECK("soft_morph_tc_qc");
    CUtensorMap tQ, tK, tG, tEV, tKD, tGT, tQT;
    MORPHO_TRY(make_tmap_3d_f16(&tQ, p.qc, MC, N, BH, MC, static_cast<uint64_t>(N) * MC, MC, kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tK, p.kc, MC, N, BH, MC, static_cast<uint64_t>(N) * MC, MC, kTile));
    MORPHO_TRY(tmap_f32_3d(&tG, x.g, HD, N, BH, 32, kTile));
    MORPHO_TRY(tmap_f32_3d(&tEV, x.evn, HD, Npad, BH, 32, kTile));
    MORPHO_TRY(tmap_f32_3d(&tKD, x.kdt, Npad, MC, BH, 32, MC));
    MORPHO_TRY(tmap_f32_3d(&tGT, x.gt, Npad, HD, BH, 32, HD));
    MORPHO_TRY(tmap_f32_3d(&tQT, x.qct, Npad, MC, BH, 32, MC));
    QArgs qa;
    qa.N = N;
    qa.Npad = Npad;
    qa.n_qtiles = n_tiles;
    qa.mask_diag = s.mask_diag ? 1 : 0;
    qa.kf2 = 2.0f * s.scale * kf;
    qa.two_scale = 2.0f * s.scale;
    qa.neg_scale = -s.scale;
    qa.mrow = p.mrow;
    qa.dq = dq;
    qa.dqb = dqb;
    qa.qb = p.qb;
    qa.sg = sg;
    qa.flag = p.smflag;
    qa.status = status;
    auto kq = sm_bwd_q_kernel<MC, HD, CAUSAL>;
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, QCfg<MC, HD>::SMEM_BYTES));
    prof_begin(stream, "soft_morph_tc_bwd_q");
    kq<<<dim3(n_tiles, BH), kThreads, QCfg<MC, HD>::SMEM_BYTES, stream>>>(tQ, tK, tG, tEV, tKD, qa);
    MORPHO_LAUNCH_CHECK("soft_morph_tc_bwd_q");
    KArgs ka;
    ka.N = N;
    ka.Npad = Npad;
    ka.H = s.H;
    ka.D = s.D;
    ka.Hp = s.Hp();
    ka.Cp = s.Cp();
    ka.n_tiles = n_tiles;
    ka.mask_diag = s.mask_diag ? 1 : 0;
    ka.kf2 = qa.kf2;
    ka.two_scale = qa.two_scale;
    ka.neg_scale = qa.neg_scale;
    ka.mrow = p.mrow;
    ka.dcat = dcat;
    ka.dk = dk;
    ka.dcb = dcb;
    ka.flag = p.smflag;
    ka.status = status;
    auto kk = sm_bwd_k_kernel<MC, HD, CAUSAL>;
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kk, cudaFuncAttributeMaxDynamicSharedMemorySize, KCfg<MC, HD>::SMEM_BYTES));
    prof_begin(stream, "soft_morph_tc_bwd_k");
    // the key side's ring stages hold KCfg::QS queries (Qc and G boxes of that many rows)
    CUtensorMap tQk, tGk;
    MORPHO_TRY(make_tmap_3d_f16(&tQk, p.qc, MC, N, BH, MC, static_cast<uint64_t>(N) * MC, MC, KCfg<MC, HD>::QS));
    MORPHO_TRY(tmap_f32_3d(&tGk, x.g, HD, N, BH, 32, KCfg<MC, HD>::QS));
    kk<<<dim3(n_tiles, BH), kThreads, KCfg<MC, HD>::SMEM_BYTES, stream>>>(tK, tQk, tEV, tGk, tGT, tQT, ka);
    MORPHO_LAUNCH_CHECK("soft_morph_tc_bwd_k");
    return MORPHO_OK;
}

}  // namespace

int launch_soft_morph_bwd_tc(const Shape& s, const ProjOut& p, const SmBwdScratch& x, const __half* dO,
                             const float* o2, float* dq, float* dqb, float* sg, float* dk, float* dcb,
                             __half* dcat, uint32_t* status, cudaStream_t st) {
    if (x.g == nullptr || x.gt == nullptr || x.evn == nullptr || x.kdt == nullptr || x.qct == nullptr ||
        p.mrow == nullptr || p.rv == nullptr || p.smflag == nullptr || p.kdq == nullptr)
        return set_error(MORPHO_ERR_INVALID, "internal: soft-morphology tensor-core backward scratch missing");
#define MORPHO_TCB_CASE(M, HDV)                                                                               \
    if (s.m == M && s.hd == HDV)                                                                              \
        return s.causal ? run_tc_bwd<M, HDV, true>(s, p, x, dO, o2, dq, dqb, sg, dk, dcb, dcat, status, st)   \
                        : run_tc_bwd<M, HDV, false>(s, p, x, dO, o2, dq, dqb, sg, dk, dcb, dcat, status, st);
    MORPHO_TCB_CASE(16, 32) MORPHO_TCB_CASE(16, 64) MORPHO_TCB_CASE(16, 128)
    MORPHO_TCB_CASE(32, 32) MORPHO_TCB_CASE(32, 64) MORPHO_TCB_CASE(32, 128)
    MORPHO_TCB_CASE(64, 32) MORPHO_TCB_CASE(64, 64) MORPHO_TCB_CASE(64, 128)
#undef MORPHO_TCB_CASE
    return set_error(MORPHO_ERR_INVALID, "soft-morphology tensor-core backward: cube_m %d, head_dim %d not supported",
                     s.m, s.hd);
}

}  // namespace morpho
