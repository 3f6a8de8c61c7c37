// softmorph_tc.cu -- the soft-morphology forward on the tensor cores (sm_100a).
//
// The score (reference csrc/cuda/morfology/soft_morph.cuh:10-61) is
//   t_ic = log2 sum_j 2^(x_ij + y_jc),   x_ij = kf2 * (k_j . qc_i),   y_jc = kf * V_jc,
// (log2 units, kf = sgn log2(e) / tau, kf2 = 2 scale kf), out_ic = sgn tau ln2 t_ic - scale qbias_i.
// The reference folds one exponential per (i, j, c) into an online log-sum-exp.  Here the
// exponential of the sum is split into the product of two exponentials,
//   sum_j 2^(x_ij + y_jc) = 2^(m_i + R_c) sum_j 2^(x_ij - m_i) 2^(y_jc - R_c),
// with m_i a running row maximum of x and R_c the column maximum of y over all keys, so the
// sum over j is a matrix product E_S . E_V of an N x N and an N x hd matrix of numbers in
// (0, 1]: one exponential per (i, j) (the softmax path's count) and a kind::tf32 MMA
// (fp32 range, 10-bit mantissa; E_V is rounded to tf32 once) instead of hd exponentials.
//
// The split is exact while the dominant term of each (i, c) is within fp32 range of its two
// stabilisers.  Every output is checked: an accumulator below 2^-90 (a dominant term that may
// have underflowed) sets a flag in device memory, and the exact CUDA-core kernel of
// softmorph.cu, launched after this one, recomputes the whole problem when the flag is set
// and returns at once otherwise.  Rows without any key (causal plus diagonal mask at query 0)
// give out = 0 and t = +inf, as in the exact kernel.
//
// Kernels:
//   ev_partial_kernel : per (b*h, 256-key block) column maxima of sgn * V
//   ev_kernel         : R_c = kf-scaled column maxima; E_V^T [B*H, hd, Npad] fp32 (keys
//                       contiguous: the K-major B operand), 0 past N
//   sm_tc_fwd_kernel  : one CTA per 128-query tile: S = qc . k^T (kind::f16, as the softmax
//                       forward), E_S = 2^(kf2 S - m) written to TMEM as fp32, acc += E_S . E_V
//                       (kind::tf32, A from TMEM), lazy rescale of acc when m grows by 2^32;
//                       12 warps (TMA producer, MMA issuer, two idle, eight exponent warps:
//                       two per TMEM lane quarter, 64 key columns each, which exchange their
//                       partial row maxima through shared memory every tile), a 4-stage ring
//                       of K codes and E_V^T tiles (2 stages at hd 128).
#include "kernels.h"
#include "sm100.cuh"

namespace morpho {
namespace {

constexpr int kTile = 128;
constexpr int kThreads = 384;  // warps 0-3: TMA, MMA, 2 idle; 4-11: two exponent warps per TMEM lane quarter
constexpr int kVBlock = 256;                 // keys per ev_partial block
constexpr float kGrowThreshold = 32.0f;      // log2 units: E_S <= 2^32, acc <= 2^32 * N
constexpr float kAccFloor = 8.0779356e-28f;  // 2^-90: below it the split may have lost the dominant term
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

inline int npad_of(int N) { return (N + kTile - 1) / kTile * kTile; }

// ---------------- E_V ----------------
// Block (bh, kb) = keys kb*256 .. +256 of one (b, h); thread = 8 consecutive channels of one
// key lane.  vpart[bh][kb][c] = max over the block's keys of sgn * V_jc (-inf if none).
template <int HD>
__global__ void __launch_bounds__(256) ev_partial_kernel(const __half* __restrict__ v, float* __restrict__ vpart,
                                                         int N, float sgn) {
    constexpr int LPR = HD / 8;      // threads per key row
    constexpr int ROWS = 256 / LPR;  // key rows per pass
    __shared__ float red[ROWS][HD];
    const int bh = blockIdx.x, kb = blockIdx.y;
    const int lr = threadIdx.x / LPR, c0 = (threadIdx.x % LPR) * 8;
    float mx[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) mx[u] = -INFINITY;
    const __half* base = v + static_cast<size_t>(bh) * N * HD;
    for (int j = kb * kVBlock + lr; j < min(N, (kb + 1) * kVBlock); j += ROWS) {
        const uint4 w = *reinterpret_cast<const uint4*>(base + static_cast<size_t>(j) * HD + c0);
        const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float2 f = __half22float2(h[u]);
            mx[2 * u] = fmaxf(mx[2 * u], sgn * f.x);
            mx[2 * u + 1] = fmaxf(mx[2 * u + 1], sgn * f.y);
        }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) red[lr][c0 + u] = mx[u];
    __syncthreads();
    if (threadIdx.x < HD) {
        float m = -INFINITY;
        for (int r = 0; r < ROWS; ++r) m = fmaxf(m, red[r][threadIdx.x]);
        vpart[(static_cast<size_t>(bh) * gridDim.y + kb) * HD + threadIdx.x] = m;
    }
}

// Block (bh, jb) = keys jb*32 .. +32.  R_c = |kf| * max_kb vpart (log2 units), then
// evt[bh][c][j] = tf32(2^(kf V_jc - R_c)) for j < N, 0 past N.  Block (bh, 0) also stores R.
template <int HD>
__global__ void __launch_bounds__(256) ev_kernel(const __half* __restrict__ v, const float* __restrict__ vpart,
                                                 int nvb, float* __restrict__ evt, float* __restrict__ rv, int N,
                                                 int Npad, float kf) {
    __shared__ float R[HD];
    __shared__ float tile[32][HD + 1];
    const int bh = blockIdx.x, j0 = blockIdx.y * 32;
    const float kf_abs = fabsf(kf);
    if (threadIdx.x < HD) {
        float m = -INFINITY;
        for (int kb = 0; kb < nvb; ++kb) m = fmaxf(m, vpart[(static_cast<size_t>(bh) * nvb + kb) * HD + threadIdx.x]);
        R[threadIdx.x] = kf_abs * m;  // max_j kf V_jc = |kf| max_j sgn V_jc
        if (blockIdx.y == 0) rv[static_cast<size_t>(bh) * HD + threadIdx.x] = kf_abs * m;
    }
    const __half* base = v + static_cast<size_t>(bh) * N * HD;
    for (int e = threadIdx.x; e < 32 * HD / 8; e += 256) {
        const int r = e / (HD / 8), c0 = (e % (HD / 8)) * 8;
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (j0 + r < N) {
            const uint4 w = *reinterpret_cast<const uint4*>(base + static_cast<size_t>(j0 + r) * HD + c0);
            const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float2 t = __half22float2(h[u]);
                f[2 * u] = t.x;
                f[2 * u + 1] = t.y;
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) tile[r][c0 + u] = f[u];
    }
    __syncthreads();
    float* dst = evt + static_cast<size_t>(bh) * HD * Npad + j0;
    for (int e = threadIdx.x; e < 32 * HD; e += 256) {
        const int c = e / 32, jj = e % 32;
        const float val = (j0 + jj < N) ? ex2(fmaf(tile[jj][c], kf, -R[c])) : 0.f;
        dst[static_cast<size_t>(c) * Npad + jj] = __uint_as_float(round_tf32(val));
    }
}

// ---------------- forward ----------------
template <int MC, int HD>
struct TcCfg {
    static constexpr int Q_BYTES = kTile * MC * 2;
    static constexpr int K_BYTES = kTile * MC * 2;
    static constexpr int EV_BYTES = HD * kTile * 4;  // four 32-key blocks of [HD rows x 128 B]
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = (Q_BYTES + 1023) / 1024 * 1024;
    static constexpr int K_STRIDE = (K_BYTES + 1023) / 1024 * 1024;
    static constexpr int ST = HD <= 64 ? 4 : 2;  // TMA ring depth (K codes + E_V^T per tile)
    static constexpr int OFF_EV = OFF_K + ST * K_STRIDE;
    static constexpr int OFF_BAR = OFF_EV + ST * EV_BYTES;
    static constexpr int SMEM_BYTES = OFF_BAR + 3072 + 1024;  // barriers, TMEM slot, 2 x 2 x 128 partial maxima; alignment
    static constexpr uint32_t TMEM_S = 0;
    static constexpr uint32_t TMEM_E = 128;
    static constexpr uint32_t TMEM_ACC = 256;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t QK_ROW_BYTES = MC * 2;
    static_assert(TMEM_ACC + HD <= TMEM_COLS, "TMEM columns");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

struct TcArgs {
    int N, Npad, H, D, n_qtiles;
    int mask_diag;
    float kf2;        // 2 scale sgn log2(e) / tau: applied to S = k . qc
    float out_mul;    // sgn tau ln2
    const float* qb;  // [BH, Npad] scale log2(e) qbias
    const float* rv;  // [BH, HD] R_c
    __half* out;      // [B, N, D] (may be null)
    float* o2;        // [BH, N, HD] t_ic (may be null)
    float* mrow;      // [BH, Npad] the final row reference m_i (for the split backward)
    uint32_t* flag;   // set when an accumulator fell below the floor
    uint32_t* status;
};

template <int MC, int HD, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    sm_tc_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmE, const TcArgs args) {
    using Cfg = TcCfg<MC, HD>;
    constexpr int kStages = Cfg::ST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    // bars: [0,S) kv_full, [S,2S) kv_empty, 2S q_full, +1 s_full, +2 e_full, +3 o_done, +4 drain, +5 s_free,
    //       +6 mx_full (both halves' partial row maxima of the tile are in shared memory)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 7);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    float* pmax = reinterpret_cast<float*>(tmem_slot + 4);  // [tile parity][half][row]

    const int warp = warp_id();
    const int lane = threadIdx.x & 31;
    const int bh = blockIdx.y;
    const int qt = CAUSAL ? (args.n_qtiles - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
    const int q0 = qt * kTile;
    const int n_kv_all = (args.N + kTile - 1) / kTile;
    const int n_kv = CAUSAL ? min(n_kv_all, qt + 1) : n_kv_all;

    const uint32_t kv_full0 = smem_u32(bars);
    const uint32_t kv_empty0 = smem_u32(bars + kStages);
    const uint32_t q_full = smem_u32(bars + 2 * kStages);
    const uint32_t s_full = q_full + 8;
    const uint32_t e_full = q_full + 16;
    const uint32_t o_done = q_full + 24;
    const uint32_t drain = q_full + 32;
    const uint32_t s_free = q_full + 40;
    const uint32_t mx_full = q_full + 48;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(kv_full0 + 8 * s, 1);
            mbar_init(kv_empty0 + 8 * s, 1);
        }
        mbar_init(q_full, 1);
        mbar_init(s_full, 1);
        mbar_init(e_full, 8);
        mbar_init(o_done, 1);
        mbar_init(drain, 1);
        mbar_init(s_free, 8);
        mbar_init(mx_full, 8);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmE);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const uint32_t sQ = smem_u32(smem + Cfg::OFF_Q);
            mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES);
            tma_load_3d(sQ, &tmQ, q_full, 0, q0, bh);
            int issued = 0;
            for (int j = 0; j < n_kv; ++j) {
                const int s = j % kStages;
                if (j >= kStages &&
                    !mbar_wait(kv_empty0 + 8 * s, ((j / kStages) & 1) ^ 1, args.status, K_SOFT_MORPH, 21)) {
                    *abort_flag = 1u;
                    break;
                }
                if (*abort_flag) break;
                const int kv0 = j * kTile;
                const uint32_t fb = kv_full0 + 8 * s;
                const uint32_t sK = smem_u32(smem + Cfg::OFF_K + s * Cfg::K_STRIDE);
                const uint32_t sE = smem_u32(smem + Cfg::OFF_EV + s * Cfg::EV_BYTES);
                mbar_arrive_expect_tx(fb, Cfg::K_BYTES + Cfg::EV_BYTES);
                tma_load_3d(sK, &tmK, fb, 0, kv0, bh);
#pragma unroll
                for (int kb = 0; kb < 4; ++kb) tma_load_3d(sE + kb * HD * 128, &tmE, fb, kv0 + 32 * kb, 0, bh);
                ++issued;
            }
            mbar_wait(q_full, 0, args.status, K_SOFT_MORPH, 22);
            if (*abort_flag) {
                for (int i = max(0, issued - kStages); i < issued; ++i)
                    mbar_wait(kv_full0 + 8 * (i % kStages), (i / kStages) & 1, args.status, K_SOFT_MORPH, 22);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc_s = make_idesc_f16(128, 128, false, false);
            constexpr uint32_t idesc_e = make_idesc_tf32(128, HD);
            constexpr uint32_t qk_sw = swizzle_code_for_row_bytes(Cfg::QK_ROW_BYTES);
            constexpr uint32_t qk_sbo = 8 * Cfg::QK_ROW_BYTES;
            const uint32_t sQ = smem_u32(smem + Cfg::OFF_Q);
            bool ok = mbar_wait(q_full, 0, args.status, K_SOFT_MORPH, 23);
            auto issue_s = [&](int j) {
                const uint32_t sK = smem_u32(smem + Cfg::OFF_K + (j % kStages) * Cfg::K_STRIDE);
#pragma unroll
                for (int ks = 0; ks < MC / 16; ++ks) {
                    const uint64_t ad = make_sdesc(sQ + ks * 32, 16, qk_sbo, qk_sw);
                    const uint64_t bd = make_sdesc(sK + ks * 32, 16, qk_sbo, qk_sw);
                    umma_ss(tmem + Cfg::TMEM_S, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
                }
                umma_commit(s_full);
            };
            if (ok && n_kv > 0) {
                ok = mbar_wait(kv_full0, 0, args.status, K_SOFT_MORPH, 24);
                if (ok) {
                    tc_fence_after();
                    issue_s(0);
                }
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                const int s = j % kStages;
                if (j + 1 < n_kv) {
                    const int s1 = (j + 1) % kStages;
                    if (!mbar_wait(s_free, j & 1, args.status, K_SOFT_MORPH, 25) ||
                        !mbar_wait(kv_full0 + 8 * s1, ((j + 1) / kStages) & 1, args.status, K_SOFT_MORPH, 26)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_s(j + 1);
                }
                if (!mbar_wait(e_full, j & 1, args.status, K_SOFT_MORPH, 27)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sE = smem_u32(smem + Cfg::OFF_EV + s * Cfg::EV_BYTES);
#pragma unroll
                for (int kb = 0; kb < 4; ++kb) {
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t bd = make_sdesc(sE + kb * HD * 128 + ks * 32, 16, 1024, SW_128);
                        umma_ts_tf32(tmem + Cfg::TMEM_ACC, tmem + Cfg::TMEM_E + kb * 32 + ks * 8, bd, idesc_e,
                                     (j > 0 || kb > 0 || ks > 0) ? 1u : 0u);
                    }
                }
                umma_commit(o_done);
                umma_commit(kv_empty0 + 8 * s);
            }
            if (!ok) {
                *abort_flag = 1u;
                umma_commit(drain);
                mbar_wait(drain, 0, args.status, K_SOFT_MORPH, 28);
            }
        }
    } else if (warp >= 4) {
        // ---------------- exponentials + epilogue (warps 4..11, two per TMEM lane quarter) ----------------
        const int quad = warp & 3;
        const int half = (warp - 4) >> 2;  // key columns half*64 .. +64, acc columns half*HD/2 .. +HD/2
        const int r = quad * 32 + lane;
        const int q = q0 + r;
        const uint32_t row_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
        const uint32_t lane_base = row_base + half * 64;
        const uint32_t acc_base = row_base + Cfg::TMEM_ACC + half * (HD / 2);
        const float kf2 = args.kf2;
        const bool pos = kf2 >= 0.f;
        float m_ref = -INFINITY;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int kv0 = j * kTile;
            if (!mbar_wait_warp(s_full, j & 1, args.status, K_SOFT_MORPH, 29)) {
                ok = false;
                break;
            }
            tc_fence_after();
            constexpr int W = kTile / 2;  // this warp's columns
            uint32_t sv[W];
#pragma unroll
            for (int c = 0; c < W; c += 32) tmem_ld32(lane_base + Cfg::TMEM_S + c, sv + c);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
            const float masked = pos ? -INFINITY : INFINITY;
            const bool need_mask = (kv0 + kTile > args.N) || ((CAUSAL || args.mask_diag) && j == qt);
            if (need_mask) {
#pragma unroll
                for (int c = 0; c < W; ++c) {
                    const int kv = kv0 + half * W + c;
                    const bool drop = kv >= args.N || (CAUSAL && kv > q) || (args.mask_diag && kv == q);
                    sv[c] = drop ? __float_as_uint(masked) : sv[c];
                }
            }
            float ms;
            {
                float a0 = u2f(sv[0]), a1 = u2f(sv[1]), a2 = u2f(sv[2]), a3 = u2f(sv[3]);
#pragma unroll
                for (int c = 4; c < W; c += 8) {
                    if (pos) {
                        a0 = fmax3(a0, u2f(sv[c]), u2f(sv[c + 1]));
                        a1 = fmax3(a1, u2f(sv[c + 2]), u2f(sv[c + 3]));
                        if (c + 4 < W) a2 = fmax3(a2, u2f(sv[c + 4]), u2f(sv[c + 5]));
                        if (c + 6 < W) a3 = fmax3(a3, u2f(sv[c + 6]), u2f(sv[c + 7]));
                    } else {
                        a0 = fmin3(a0, u2f(sv[c]), u2f(sv[c + 1]));
                        a1 = fmin3(a1, u2f(sv[c + 2]), u2f(sv[c + 3]));
                        if (c + 4 < W) a2 = fmin3(a2, u2f(sv[c + 4]), u2f(sv[c + 5]));
                        if (c + 6 < W) a3 = fmin3(a3, u2f(sv[c + 6]), u2f(sv[c + 7]));
                    }
                }
                ms = pos ? fmax3(a0, a1, fmaxf(a2, a3)) : fmin3(a0, a1, fminf(a2, a3));
            }
            // the row's extreme over both halves: exchange through shared memory (double-buffered
            // by tile parity, so a warp one tile ahead never overwrites a value still to be read)
            {
                float* slot = pmax + (j & 1) * 2 * kTile;
                slot[half * kTile + r] = ms;
                __syncwarp();
                if (lane == 0) mbar_arrive(mx_full);
                if (!mbar_wait_warp(mx_full, j & 1, args.status, K_SOFT_MORPH, 32)) {
                    ok = false;
                    break;
                }
                const float other = slot[(1 - half) * kTile + r];
                ms = pos ? fmaxf(ms, other) : fminf(ms, other);
            }
            const float mt = kf2 * ms;  // -inf when every key of the tile is masked
            const bool grow = mt > m_ref + kGrowThreshold;
            const float m_new = grow ? mt : m_ref;
            const float alpha = grow ? ex2(m_ref - m_new) : 1.0f;  // 0 while m_ref is -inf
            m_ref = m_new;
            const float nm = m_ref == -INFINITY ? 0.f : -m_ref;
            // E_S = 2^(kf2 S - m) in fp32, in place (masked keys give 0); they overlap the
            // previous E_S . E_V, which still reads the E columns
#pragma unroll
            for (int c = 0; c < W; ++c) sv[c] = __float_as_uint(ex2(fmaf(u2f(sv[c]), kf2, nm)));
            if (j > 0) {
                if (!mbar_wait_warp(o_done, (j - 1) & 1, args.status, K_SOFT_MORPH, 30)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                    for (int c = 0; c < HD / 2; c += 16) {
                        uint32_t rr[16];
                        tmem_ld16(acc_base + c, rr);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) rr[i] = __float_as_uint(u2f(rr[i]) * alpha);
                        tmem_st16(acc_base + c, rr);
                    }
                    tmem_st_wait();
                }
            }
#pragma unroll
            for (int c = 0; c < W; c += 16) tmem_st16(lane_base + Cfg::TMEM_E + c, sv + c);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(e_full);
        }
        // ---- epilogue: t = m + R + log2(acc) -> o2, out
        if (ok && n_kv > 0 && mbar_wait_warp(o_done, (n_kv - 1) & 1, args.status, K_SOFT_MORPH, 31)) {
            tc_fence_after();
            const int b = bh / args.H;
            const int h = bh - b * args.H;
            const bool live = q < args.N;
            const bool dead = m_ref == -INFINITY;  // no key at all: out 0, t +inf
            const float qbl = live ? kLn2 * args.qb[static_cast<size_t>(bh) * args.Npad + q] : 0.f;
            const float* R = args.rv + static_cast<size_t>(bh) * HD + half * (HD / 2);
            __half* orow = args.out == nullptr
                               ? nullptr
                               : args.out + (static_cast<size_t>(b) * args.N + q) * args.D + h * HD + half * (HD / 2);
            float* o2row =
                args.o2 == nullptr ? nullptr : args.o2 + (static_cast<size_t>(bh) * args.N + q) * HD + half * (HD / 2);
            bool low = false;
#pragma unroll
            for (int c = 0; c < HD / 2; c += 16) {
                uint32_t rr[16];
                tmem_ld16(acc_base + c, rr);
                tmem_ld_wait();
                float t[16];
                uint32_t pk[8];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float acc = u2f(rr[i]);
                    low |= !(acc >= kAccFloor);
                    t[i] = dead ? INFINITY : m_ref + R[c + i] + log2f(acc);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    pk[i] = pack_half2(dead ? 0.f : args.out_mul * t[2 * i] - qbl,
                                       dead ? 0.f : args.out_mul * t[2 * i + 1] - qbl);
                if (live && orow != nullptr) {
                    uint4* dst = reinterpret_cast<uint4*>(orow + c);
                    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
                if (live && o2row != nullptr) {
                    float4* d2 = reinterpret_cast<float4*>(o2row + c);
#pragma unroll
                    for (int i = 0; i < 4; ++i) d2[i] = make_float4(t[4 * i], t[4 * i + 1], t[4 * i + 2], t[4 * i + 3]);
                }
            }
            if (live && half == 0) args.mrow[static_cast<size_t>(bh) * args.Npad + q] = m_ref;
            if (live && !dead && low) atomicOr(args.flag, 1u);
        } else if (!ok) {
            *abort_flag = 1u;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

template <int MC, int HD, bool CAUSAL>
int run_tc_fwd(const Shape& s, const ProjOut& p, __half* out, float* o2, uint32_t* status, cudaStream_t stream) {
    using Cfg = TcCfg<MC, HD>;
    const int BH = s.B * s.H;
    const int Npad = npad_of(s.N);
    const int nvb = (s.N + kVBlock - 1) / kVBlock;
    const float sgn = s.score == kScoreErosion ? -1.0f : 1.0f;
    const float kf = sgn * kLog2e / s.tau;
    MORPHO_CUDA_TRY(cudaMemsetAsync(p.smflag, 0, sizeof(uint32_t), stream));
    prof_begin(stream, "soft_morph_ev_partial");
    ev_partial_kernel<HD><<<dim3(BH, nvb), 256, 0, stream>>>(p.v, p.vpart, s.N, sgn);
    MORPHO_LAUNCH_CHECK("soft_morph_ev_partial");
    prof_begin(stream, "soft_morph_ev");
    ev_kernel<HD><<<dim3(BH, Npad / 32), 256, 0, stream>>>(p.v, p.vpart, nvb, p.evt, p.rv, s.N, Npad, kf);
    MORPHO_LAUNCH_CHECK("soft_morph_ev");
    CUtensorMap tQ, tK, tE;
    MORPHO_TRY(make_tmap_3d_f16(&tQ, p.qc, MC, s.N, BH, MC, static_cast<uint64_t>(s.N) * MC, MC, kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tK, p.kc, MC, s.N, BH, MC, static_cast<uint64_t>(s.N) * MC, MC, kTile));
    {
        const uint64_t dims[3] = {static_cast<uint64_t>(Npad), static_cast<uint64_t>(HD), static_cast<uint64_t>(BH)};
        const uint64_t strides[2] = {static_cast<uint64_t>(Npad) * 4, static_cast<uint64_t>(Npad) * HD * 4};
        const uint32_t box[3] = {32, HD, 1};
        MORPHO_TRY(make_tmap(&tE, p.evt, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B));
    }
    TcArgs a;
    a.N = s.N;
    a.Npad = Npad;
    a.H = s.H;
    a.D = s.D;
    a.n_qtiles = Npad / kTile;
    a.mask_diag = s.mask_diag ? 1 : 0;
    a.kf2 = 2.0f * s.scale * kf;
    a.out_mul = sgn * s.tau * kLn2;
    a.qb = p.qb;
    a.rv = p.rv;
    a.out = out;
    a.o2 = o2;
    a.flag = p.smflag;
    a.mrow = p.mrow;
    a.status = status;
    auto kern = sm_tc_fwd_kernel<MC, HD, CAUSAL>;
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    prof_begin(stream, "soft_morph_tc_fwd");
    kern<<<dim3(a.n_qtiles, BH), kThreads, Cfg::SMEM_BYTES, stream>>>(tQ, tK, tE, a);
    MORPHO_LAUNCH_CHECK("soft_morph_tc_fwd");
    return MORPHO_OK;
}

template <int MC, int HD>
int run_tc_fwd_c(const Shape& s, const ProjOut& p, __half* out, float* o2, uint32_t* status, cudaStream_t st) {
    return s.causal ? run_tc_fwd<MC, HD, true>(s, p, out, o2, status, st)
                    : run_tc_fwd<MC, HD, false>(s, p, out, o2, status, st);
}

}  // namespace

int launch_soft_morph_fwd_tc(const DeviceInfo& dev, const Shape& s, const ProjOut& p, __half* out, float* o2,
                             cudaStream_t st) {
    if (p.evt == nullptr || p.rv == nullptr || p.vpart == nullptr || p.smflag == nullptr || p.mrow == nullptr)
        return set_error(MORPHO_ERR_INVALID, "internal: soft-morphology forward scratch missing");
    if (soft_morph_exact_only()) {
        // exact kernels only; the flag is set so that a backward run without the switch also
        // takes the exact pair (this forward leaves no m_i / R_c behind)
        MORPHO_CUDA_TRY(cudaMemsetAsync(p.smflag, 0xFF, sizeof(uint32_t), st));
        return launch_soft_morph_fwd(s, p, out, o2, nullptr, st);
    }
    int rc = MORPHO_OK;
    bool matched = false;
#define MORPHO_TC_CASE(M, HDV)                                    \
    if (s.m == M && s.hd == HDV) {                                \
        matched = true;                                           \
        rc = run_tc_fwd_c<M, HDV>(s, p, out, o2, dev.status, st); \
    }
    MORPHO_TC_CASE(16, 32) MORPHO_TC_CASE(16, 64) MORPHO_TC_CASE(16, 128)
    MORPHO_TC_CASE(32, 32) MORPHO_TC_CASE(32, 64) MORPHO_TC_CASE(32, 128)
    MORPHO_TC_CASE(64, 32) MORPHO_TC_CASE(64, 64) MORPHO_TC_CASE(64, 128)
#undef MORPHO_TC_CASE
    if (!matched)
        return set_error(MORPHO_ERR_INVALID, "soft-morphology score: cube_m %d, head_dim %d not supported", s.m, s.hd);
    if (rc != MORPHO_OK) return rc;
    // the exact kernel recomputes everything only when an accumulator was flagged
    return launch_soft_morph_fwd(s, p, out, o2, p.smflag, st);
}

}  // namespace morpho
