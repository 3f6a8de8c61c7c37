// attn_fwd.cu -- MorphoAttention forward on sm_100a over the projected codes.
//
// One CTA = one 128-row query tile of one (batch, head).  The reference re-projects
// K and V from x for every (query block, KV tile) pair (attention.cu:91-111); here the
// codes and V come from the projection GEMM, and each KV tile is one TMA box.
//
// Per KV tile j (128 keys):
//   MMA warp   : S = Qc . Kc^T   (M=128, N=128, K=cube_m)         -> TMEM cols [0,128)
//                with centered query codes, so S = q.k - cb_j/2 (cb_j = sum_c gate_q k_jc)
//   softmax    : t = 2*scale*log2e * S = 2*scale*log2e*q.k - cb'_j (attention.cu:125 with
//                the row-constant query bias moved into lse), masks, row max,
//                p = 2^(t - m) -> fp16 P                          -> TMEM cols [128,192)
//   MMA warp   : O += P . V_j    (A = P from TMEM, B = V MN-major) -> TMEM cols [192, ..)
// The running max is rescaled lazily: O and l are only corrected when the max grows by
// more than 2^8, so P stays <= 256 (exact in fp16 range) and most tiles skip the O
// round trip.  The reference keeps O in shared memory and rescales it every tile
// (attention.cu:166-169).
//
// lse (log2 domain, attention.cu:186) = m + log2(l) - qb', qb' = scale*log2e*qbias.
//
// Warps (256 threads, two warpgroups): 0 = TMA producer, 1 = TMEM owner + MMA issuer,
// 2-3 idle, 4..7 = softmax and epilogue (warp w owns TMEM lanes / query rows
// 32*(w%4) .. +31).  setmaxnreg moves registers from the first to the second warpgroup.
#include "kernels.h"
#include "sm100.cuh"

namespace morpho {
namespace {

constexpr int kFwdThreads = 256;
// Register split (256 threads x 128 at launch, two CTAs per SM): producer/MMA warpgroup
// 56, softmax warpgroup 200; 128*56 + 128*200 = 256*128.
constexpr uint32_t kRegsProducer = 56;
constexpr uint32_t kRegsSoftmax = 200;
static_assert(128 * kRegsProducer + 128 * kRegsSoftmax == kFwdThreads * 128, "register split");
constexpr int kTile = 128;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int MC, int HD>
struct FwdCfg {
    // hd = 128: P (fp16, 64 columns) is written over the first half of S, which the softmax warps
    // hold in registers by then, so S + O fit 256 TMEM columns and, with two K/V stages and no
    // alignment slack, two CTAs share an SM as they do at hd <= 64.  S(j+1) is then issued after
    // P.V(j) (in issue order it cannot overwrite P(j) before that MMA read it) instead of as soon as
    // S(j) is read; the other CTA of the SM covers that wait.
    static constexpr bool P_IN_S = HD > 64;
    static constexpr int KV_STAGES = P_IN_S ? 2 : 3;
    static constexpr int Q_BYTES = kTile * MC * 2;
    static constexpr int K_BYTES = kTile * MC * 2;
    static constexpr int V_BYTES = kTile * HD * 2;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = (Q_BYTES + 1023) / 1024 * 1024;
    static constexpr int K_STRIDE = (K_BYTES + 1023) / 1024 * 1024;
    static constexpr int OFF_V = OFF_K + KV_STAGES * K_STRIDE;
    static constexpr int OFF_BAR = OFF_V + KV_STAGES * V_BYTES;
    static constexpr int USED = OFF_BAR + 256;
    // (P_IN_S: the dynamic shared memory is declared 1024-byte aligned, checked at run time,
    // instead of 1 KB of slack, so that two CTAs of m = 64 fit an SM)
    static constexpr int SMEM_BYTES = P_IN_S ? USED : USED + 1024;
    static_assert(!P_IN_S || 2 * (SMEM_BYTES + 1024) <= 233472, "two CTAs per SM");
    static constexpr uint32_t TMEM_S = 0;
    static constexpr uint32_t TMEM_P = P_IN_S ? 0 : 128;
    static constexpr uint32_t TMEM_O = P_IN_S ? 128 : 192;
    static constexpr uint32_t TMEM_COLS = 256;
    static constexpr uint32_t QK_ROW_BYTES = MC * 2;
    static constexpr uint32_t V_ROW_BYTES = (HD > 64 ? 64 : HD) * 2;
};

struct FwdArgs {
    int N, Npad, H, D, n_qtiles;
    int BH, band;   // causal launch order (causal_order)
    int mask_diag;  // also drop key j == query i
    float c2;  // 2 * scale * log2(e)
    const float* qb;
    __half* out;
    float* lse;
    uint32_t* status;
};

template <int MC, int HD, bool CAUSAL>
__global__ void __launch_bounds__(kFwdThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FwdArgs args) {
    using Cfg = FwdCfg<MC, HD>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (Cfg::P_IN_S && (smem_u32(smem_raw) & 1023u) != 0u) {  // no slack to align in: refuse
        if (threadIdx.x == 0) report_timeout(args.status, K_ATTN_FWD, 30);
        return;
    }
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    // bars: [0,S) kv_full, [S,2S) kv_empty, 2S q_full, 2S+1 s_full, 2S+2 p_full, 2S+3 o_done, 2S+4 drain,
    //       2S+5 s_free
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * Cfg::KV_STAGES + 6);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int warp = warp_id();
    const int lane = threadIdx.x & 31;
    int qt, bh;
    if (CAUSAL) {  // query tile qt meets qt + 1 key tiles: heaviest (last) first
        int t;
        causal_order(static_cast<int>(blockIdx.x), args.n_qtiles, args.BH, args.band, t, bh);
        qt = args.n_qtiles - 1 - t;
    } else {
        qt = static_cast<int>(blockIdx.x);
        bh = static_cast<int>(blockIdx.y);
    }
    const int q0 = qt * kTile;
    const int n_kv_all = (args.N + kTile - 1) / kTile;
    const int n_kv = CAUSAL ? min(n_kv_all, qt + 1) : n_kv_all;

    const uint32_t kv_full0 = smem_u32(bars);
    const uint32_t kv_empty0 = smem_u32(bars + Cfg::KV_STAGES);
    const uint32_t q_full = smem_u32(bars + 2 * Cfg::KV_STAGES);
    const uint32_t s_full = q_full + 8;
    const uint32_t p_full = q_full + 16;
    const uint32_t o_done = q_full + 24;
    const uint32_t drain = q_full + 32;
    const uint32_t s_free = q_full + 40;  // the softmax warps hold S_j in registers

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::KV_STAGES; ++s) {
            mbar_init(kv_full0 + 8 * s, 1);
            mbar_init(kv_empty0 + 8 * s, 1);  // released by the MMA commit after P.V
        }
        mbar_init(q_full, 1);
        mbar_init(s_full, 1);
        mbar_init(p_full, 4);
        mbar_init(o_done, 1);
        mbar_init(drain, 1);
        mbar_init(s_free, 4);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
      regs_dec<kRegsProducer>();
      if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const uint32_t sQ = smem_u32(smem + Cfg::OFF_Q);
            mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES);
            tma_load_3d(sQ, &tmQ, q_full, 0, q0, bh);
            int issued = 0;
            for (int j = 0; j < n_kv; ++j) {
                const int s = j % Cfg::KV_STAGES;
                if (j >= Cfg::KV_STAGES &&
                    !mbar_wait(kv_empty0 + 8 * s, ((j / Cfg::KV_STAGES) & 1) ^ 1, args.status, K_ATTN_FWD, 1)) {
                    *abort_flag = 1u;
                    break;
                }
                if (*abort_flag) break;
                const int kv0 = j * kTile;
                const uint32_t fb = kv_full0 + 8 * s;
                const uint32_t sK = smem_u32(smem + Cfg::OFF_K + s * Cfg::K_STRIDE);
                const uint32_t sV = smem_u32(smem + Cfg::OFF_V + s * Cfg::V_BYTES);
                mbar_arrive_expect_tx(fb, Cfg::K_BYTES + Cfg::V_BYTES);
                tma_load_3d(sK, &tmK, fb, 0, kv0, bh);
                if (HD > 64) {
                    tma_load_3d(sV, &tmV, fb, 0, kv0, bh);
                    tma_load_3d(sV + kTile * 128, &tmV, fb, 64, kv0, bh);
                } else {
                    tma_load_3d(sV, &tmV, fb, 0, kv0, bh);
                }
                ++issued;
            }
            // Bounded drain of loads still in flight (abort path, and the Q tile).
            mbar_wait(q_full, 0, args.status, K_ATTN_FWD, 2);
            if (*abort_flag) {
                for (int i = max(0, issued - Cfg::KV_STAGES); i < issued; ++i)
                    mbar_wait(kv_full0 + 8 * (i % Cfg::KV_STAGES), (i / Cfg::KV_STAGES) & 1, args.status, K_ATTN_FWD, 2);
            }
        }
      } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        // The whole warp runs this loop (warp-uniform control flow and descriptor arithmetic);
        // elect.sync inside umma_*_w / umma_commit_w lets one lane issue each instruction.
        {
            constexpr uint32_t idesc_s = make_idesc_f16(128, 128, false, false);
            constexpr uint32_t idesc_pv = make_idesc_f16(128, HD, false, true);
            constexpr uint32_t qk_sw = swizzle_code_for_row_bytes(Cfg::QK_ROW_BYTES);
            constexpr uint32_t qk_sbo = 8 * Cfg::QK_ROW_BYTES;
            constexpr uint32_t v_sw = swizzle_code_for_row_bytes(Cfg::V_ROW_BYTES);
            constexpr uint32_t v_sbo = 8 * Cfg::V_ROW_BYTES;
            const uint32_t sQ = smem_u32(smem + Cfg::OFF_Q);
            bool ok = mbar_wait_warp(q_full, 0, args.status, K_ATTN_FWD, 3);
            auto issue_s = [&](int j) {
                const uint32_t sK = smem_u32(smem + Cfg::OFF_K + (j % Cfg::KV_STAGES) * Cfg::K_STRIDE);
#pragma unroll
                for (int ks = 0; ks < MC / 16; ++ks) {
                    const uint64_t ad = make_sdesc(sQ + ks * 32, 16, qk_sbo, qk_sw);
                    const uint64_t bd = make_sdesc(sK + ks * 32, 16, qk_sbo, qk_sw);
                    umma_ss_w(tmem + Cfg::TMEM_S, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
                }
                umma_commit_w(s_full);
            };
            if (ok && n_kv > 0) {
                ok = mbar_wait_warp(kv_full0, 0, args.status, K_ATTN_FWD, 4);
                if (ok) {
                    tc_fence_after();
                    issue_s(0);
                }
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                const int s = j % Cfg::KV_STAGES;
                // S_{j+1} as soon as the softmax warps have read S_j (its columns are free),
                // so the next scores are ready when they finish P_j
                if (!Cfg::P_IN_S && j + 1 < n_kv) {
                    const int s1 = (j + 1) % Cfg::KV_STAGES;
                    // (no abort-flag read here: every shared-memory probe of the MMA thread stalls
                    // it while MMAs are in flight; a failure elsewhere ends its bounded waits)
                    if (!mbar_wait_warp(s_free, j & 1, args.status, K_ATTN_FWD, 12) ||
                        !mbar_wait_warp(kv_full0 + 8 * s1, ((j + 1) / Cfg::KV_STAGES) & 1, args.status, K_ATTN_FWD, 6)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_s(j + 1);
                }
                if (!mbar_wait_warp(p_full, j & 1, args.status, K_ATTN_FWD, 5)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sV = smem_u32(smem + Cfg::OFF_V + s * Cfg::V_BYTES);
#pragma unroll
                for (int ks = 0; ks < kTile / 16; ++ks) {
                    const uint64_t bd = make_sdesc(sV + ks * 16 * Cfg::V_ROW_BYTES, kTile * 128, v_sbo, v_sw);
                    umma_ts_w(tmem + Cfg::TMEM_O, tmem + Cfg::TMEM_P + ks * 8, bd, idesc_pv,
                            (j > 0 || ks > 0) ? 1u : 0u);
                }
                umma_commit_w(o_done);
                umma_commit_w(kv_empty0 + 8 * s);
                if (Cfg::P_IN_S && j + 1 < n_kv) {  // S(j+1) over P(j), which P.V(j) has read (issue order)
                    const int s1 = (j + 1) % Cfg::KV_STAGES;
                    if (!mbar_wait_warp(kv_full0 + 8 * s1, ((j + 1) / Cfg::KV_STAGES) & 1, args.status, K_ATTN_FWD, 6)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_s(j + 1);
                }
            }
            if (!ok) {
                *abort_flag = 1u;
                umma_commit_w(drain);
                mbar_wait_warp(drain, 0, args.status, K_ATTN_FWD, 7);
            }
        }
      }
    } else {
        regs_inc<kRegsSoftmax>();
        // ---------------- softmax + epilogue (warps 4..7) ----------------
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // query row within the tile
        const int q = q0 + r;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
        const float c2 = args.c2;
        const bool pos = c2 >= 0.f;
        float m_ref = -INFINITY;
        float l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int kv0 = j * kTile;
            // (S_j is the only input: the MMA thread already waited for the K/V tile)
            if (!mbar_wait_warp(s_full, j & 1, args.status, K_ATTN_FWD, 8)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // S = q.k - cb/2 for the 128 keys of this tile: all four TMEM loads in flight
            uint32_t sv[kTile];
#pragma unroll
            for (int c = 0; c < kTile; c += 32) tmem_ld32(lane_base + Cfg::TMEM_S + c, sv + c);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
            // t = c2 * S.  The row max of t is c2 * (max or min of S, by the sign of c2);
            // masked keys get -inf / +inf so that c2 * S - m is -inf for them.
            const float masked = pos ? -INFINITY : INFINITY;
            const bool need_mask = (kv0 + kTile > args.N) || ((CAUSAL || args.mask_diag) && j == qt);
            if (need_mask) {
#pragma unroll
                for (int c = 0; c < kTile; ++c) {
                    const int kv = kv0 + c;
                    const bool drop = kv >= args.N || (CAUSAL && kv > q) || (args.mask_diag && kv == q);
                    sv[c] = drop ? __float_as_uint(masked) : sv[c];
                }
            }
            // row max (min) with the three-input max.f32 / min.f32 of sm_100: four chains of 16
            float ms;
            {
                float a0 = u2f(sv[0]), a1 = u2f(sv[1]), a2 = u2f(sv[2]), a3 = u2f(sv[3]);
                if (pos) {
#pragma unroll
                    for (int c = 4; c < kTile; c += 8) {
                        a0 = fmax3(a0, u2f(sv[c]), u2f(sv[c + 1]));
                        a1 = fmax3(a1, u2f(sv[c + 2]), u2f(sv[c + 3]));
                        if (c + 4 < kTile) a2 = fmax3(a2, u2f(sv[c + 4]), u2f(sv[c + 5]));
                        if (c + 6 < kTile) a3 = fmax3(a3, u2f(sv[c + 6]), u2f(sv[c + 7]));
                    }
                    ms = fmax3(a0, a1, fmaxf(a2, a3));
                } else {
#pragma unroll
                    for (int c = 4; c < kTile; c += 8) {
                        a0 = fmin3(a0, u2f(sv[c]), u2f(sv[c + 1]));
                        a1 = fmin3(a1, u2f(sv[c + 2]), u2f(sv[c + 3]));
                        if (c + 4 < kTile) a2 = fmin3(a2, u2f(sv[c + 4]), u2f(sv[c + 5]));
                        if (c + 6 < kTile) a3 = fmin3(a3, u2f(sv[c + 6]), u2f(sv[c + 7]));
                    }
                    ms = fmin3(a0, a1, fminf(a2, a3));
                }
            }
            const float mt = c2 * ms;
            // Lazy rescale: move the reference max only when the row max grew by > 2^8.
            const bool grow = mt > m_ref + kRescaleThreshold;
            const float m_new = grow ? mt : m_ref;
            const float alpha = grow ? ex2(m_ref - m_new) : 1.0f;  // 0 when m_ref = -inf
            l *= alpha;
            m_ref = m_new;
            // The exponentials first, packed in place into sv[0, 64): they only need the new
            // reference max, so they overlap the previous P.V MMA, which still reads P and O.
            // m_ref is -inf only while every key of the row so far was masked (causal plus
            // diagonal mask at query 0): then all of this tile's P are 0, and l stays 0.
            float lsum = 0.f;
            const float nm = m_ref == -INFINITY ? 0.f : -m_ref;
#pragma unroll
            for (int i = 0; i < kTile / 2; ++i) {
                const float p0 = ex2(fmaf(u2f(sv[2 * i]), c2, nm));
                const float p1 = ex2(fmaf(u2f(sv[2 * i + 1]), c2, nm));
                lsum += p0 + p1;
                sv[i] = pack_half2(p0, p1);
            }
            l += lsum;
            if (j > 0) {
                // P and O are both used by the previous P.V MMA: wait for it.
                if (!mbar_wait_warp(o_done, (j - 1) & 1, args.status, K_ATTN_FWD, 10)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                    for (int c = 0; c < HD; c += 16) {
                        uint32_t rr[16];
                        tmem_ld16(lane_base + Cfg::TMEM_O + c, rr);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) rr[i] = __float_as_uint(u2f(rr[i]) * alpha);
                        tmem_st16(lane_base + Cfg::TMEM_O + c, rr);
                    }
                    tmem_st_wait();
                }
            }
#pragma unroll
            for (int c = 0; c < kTile / 2; c += 16) tmem_st16(lane_base + Cfg::TMEM_P + c, sv + c);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        // ---- epilogue: O / l -> out, lse
        if (ok && n_kv > 0 && mbar_wait_warp(o_done, (n_kv - 1) & 1, args.status, K_ATTN_FWD, 11)) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            const int b = bh / args.H;
            const int h = bh - b * args.H;
            __half* orow = args.out + (static_cast<size_t>(b) * args.N + q) * args.D + h * HD;
#pragma unroll
            for (int c = 0; c < HD; c += 16) {
                uint32_t rr[16];
                tmem_ld16(lane_base + Cfg::TMEM_O + c, rr);
                tmem_ld_wait();
                if (q < args.N) {
                    uint4* dst = reinterpret_cast<uint4*>(orow + c);
                    dst[0] = make_uint4(pack_half2(u2f(rr[0]) * inv, u2f(rr[1]) * inv),
                                        pack_half2(u2f(rr[2]) * inv, u2f(rr[3]) * inv),
                                        pack_half2(u2f(rr[4]) * inv, u2f(rr[5]) * inv),
                                        pack_half2(u2f(rr[6]) * inv, u2f(rr[7]) * inv));
                    dst[1] = make_uint4(pack_half2(u2f(rr[8]) * inv, u2f(rr[9]) * inv),
                                        pack_half2(u2f(rr[10]) * inv, u2f(rr[11]) * inv),
                                        pack_half2(u2f(rr[12]) * inv, u2f(rr[13]) * inv),
                                        pack_half2(u2f(rr[14]) * inv, u2f(rr[15]) * inv));
                }
            }
            if (q < args.N) {
                const float qb = args.qb[static_cast<size_t>(bh) * args.Npad + q];
                args.lse[static_cast<size_t>(bh) * args.N + q] = l > 0.f ? m_ref + log2f(l) - qb : -3.402823466e38f;
            }
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
int run_fwd(const DeviceInfo& dev, const Shape& s, const ProjOut& p, __half* out, float* lse, cudaStream_t stream) {
    using Cfg = FwdCfg<MC, HD>;
    const int BH = s.B * s.H;
    const int Npad = (s.N + kTile - 1) / kTile * kTile;
    CUtensorMap tQ, tK, tV;
    MORPHO_TRY(make_tmap_3d_f16(&tQ, p.qc, MC, s.N, BH, MC, static_cast<uint64_t>(s.N) * MC, MC, kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tK, p.kc, MC, s.N, BH, MC, static_cast<uint64_t>(s.N) * MC, MC, kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tV, p.v, HD, s.N, BH, HD, static_cast<uint64_t>(s.N) * HD, HD > 64 ? 64 : HD,
                                kTile));
    FwdArgs a;
    a.N = s.N;
    a.Npad = Npad;
    a.H = s.H;
    a.D = s.D;
    a.n_qtiles = Npad / kTile;
    a.mask_diag = s.mask_diag ? 1 : 0;
    a.c2 = 2.0f * s.scale * kLog2e;
    a.qb = p.qb;
    a.out = out;
    a.lse = lse;
    a.status = dev.status;
    auto kern = attn_fwd_kernel<MC, HD, CAUSAL>;
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    a.BH = BH;
    a.band = causal_band(static_cast<long long>(s.N) * (2 * MC + 2 * HD), BH, a.n_qtiles);
    const dim3 grid = CAUSAL ? dim3(a.n_qtiles * BH, 1) : dim3(a.n_qtiles, BH);
    prof_begin(stream, "attn_fwd");
    kern<<<grid, kFwdThreads, Cfg::SMEM_BYTES, stream>>>(tQ, tK, tV, a);
    MORPHO_LAUNCH_CHECK("attn_fwd");
    return MORPHO_OK;
}

template <int MC, int HD>
int run_fwd_c(const DeviceInfo& dev, const Shape& s, const ProjOut& p, __half* out, float* lse, cudaStream_t st) {
    return s.causal ? run_fwd<MC, HD, true>(dev, s, p, out, lse, st) : run_fwd<MC, HD, false>(dev, s, p, out, lse, st);
}

template <int MC>
int run_fwd_hd(const DeviceInfo& dev, const Shape& s, const ProjOut& p, __half* out, float* lse, cudaStream_t st) {
    switch (s.hd) {
        case 32: return run_fwd_c<MC, 32>(dev, s, p, out, lse, st);
        case 64: return run_fwd_c<MC, 64>(dev, s, p, out, lse, st);
        case 128: return run_fwd_c<MC, 128>(dev, s, p, out, lse, st);
        default: return set_error(MORPHO_ERR_INVALID, "head_dim %d not supported (32, 64 or 128)", s.hd);
    }
}

}  // namespace

int launch_attn_fwd(const DeviceInfo& dev, const Shape& s, const ProjOut& p, __half* out, float* lse,
                    cudaStream_t stream) {
    switch (s.m) {
        case 16: return run_fwd_hd<16>(dev, s, p, out, lse, stream);
        case 32: return run_fwd_hd<32>(dev, s, p, out, lse, stream);
        case 64: return run_fwd_hd<64>(dev, s, p, out, lse, stream);
        default: return set_error(MORPHO_ERR_INVALID, "cube_m %d not supported (16, 32 or 64)", s.m);
    }
}

}  // namespace morpho
