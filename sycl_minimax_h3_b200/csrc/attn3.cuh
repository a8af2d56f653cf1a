// attn3.cuh - the SageAttention v1 core for sm_100a: two 128-row query tiles per CTA (256 query rows), each with its
// own S buffer, softmax warpgroup and O accumulator in TMEM; every key tile's scores are computed in two halves of 64
// keys so that the next tile's scores are mostly ready before the softmax of this one ends.
//
// Warps: 0 TMA producer of Q0, Q1 (once) and the ring of K tiles; 1 TMEM owner and MMA issuer of query tile 0, 3 MMA
// issuer of tile 1 (each whole warp runs its loop, elect.sync picks the issuing lane); 2 TMA producer of the ring of
// half V tiles; 4-7 softmax of query tile 0, 8-11 of tile 1 (one thread per query row; warp w reads TMEM lane quarter
// w % 4). The same kernel, instantiated with I8 = false, is the fp16 SDPA (fp16 Q.K^T, fp32 scores, one scale).
// TMEM (512 columns): S0 0-127, S1 128-255, O0 256-383, O1 384-511 (64-wide heads: O0 256-319, O1 320-383). In S_t,
// columns 0-63 hold the scores of keys 0-63 of a key tile (S_lo) and then P_t of all 128 keys (half, two per column);
// columns 64-127 hold the scores of keys 64-127 (S_hi).
//
// The chain of one query tile t and key tile j (int8 Q.K^T on tcgen05 kind::i8 into int32, P.V on kind::f16):
//   1. the softmax loads S_hi(j) and at once lets the MMA thread issue S_hi(j+1) = Q_t.K_{j+1}[64:128)^T into the same
//      columns (hi_free);
//   2. it takes the max of S_hi(j) (per row, a lazily moved running max), its exps, and keeps P_hi in registers;
//   3. it loads S_lo(j) (issued after P_t(j-1).V_{j-1}, which read columns 0-63), takes its max, and if that moves
//      the running max, scales the P_hi registers down (rare after the first tiles); then the exps of S_lo;
//   4. it stores P(j) into columns 0-63, rescales O_t where the max moved, and hands P(j) over (p_full);
//   5. the MMA thread issues O_t += P_t(j).V_j, then S_lo(j+1) = Q_t.K_{j+1}[0:64)^T into columns 0-63.
// Steps 1-2 of tile j+1 overlap step 5 of tile j, so the softmax warps do not wait for P.V and the next Q.K^T;
// the two query tiles' warps share each SM sub-partition and keep its MUFU unit busy together.
// A commit counts every MMA issued before it: when S_lo_t(j) is complete, O_t holds the sum up to key tile j-1.
//
// Softmax arithmetic per element (log2 units): int32 x + bits(1.5*2^23) is the float 1.5*2^23 + x (exact for
// |x| < 2^22; |x| <= 128*127*127), one FFMA applies the dequantisation scale qs*ks*scale*log2(e) and subtracts the
// running max: arg = (1.5*2^23 + x)*c - (1.5*2^23*c + m); ex2.approx gives p, rounded to half for P. The running max
// moves only when a half tile's max passes it by more than 8 (weights up to 2^8); then l, O and the P_hi registers
// are scaled by 2^(m_old - m_new).
#pragma once
#include <cstdlib>

#include "attn_common.cuh"

namespace h3 {

// The int32 bits that become -inf once the bias is added: keys past S.
constexpr uint32_t kMaskedRaw = 0xFF800000u - kBias;

// I8: the Sage core (int8 Q, K with per-block scales). !I8: the fp16 SDPA (fp16 Q, K; fp32 scores; one scale) in the
// same structure, for the sequences below the Sage threshold. HD: the head width the kernel computes, 128, or 64 for
// the fp16 SDPA of heads up to 64 wide (the VAE's): Q.K^T with K = 64, P.V with N = 64, 16 KB tiles and deeper rings,
// O in 64 TMEM columns per tile.
template <bool I8, int HD = kHeadDim>
struct Sage3Cfg {
    static_assert(HD == kHeadDim || (!I8 && HD == 64), "64-wide heads on the fp16 path only");
    static constexpr int NQ = 2;                             // query tiles per CTA
    static constexpr int CB_BYTES = 128 * 128;               // one column block: 128 rows x 128 bytes, 128-byte swizzle
    static constexpr int NCB = I8 ? 1 : HD / 64;             // column blocks of a Q or K tile (int8: 128 features)
    static constexpr int TILE_B = NCB * CB_BYTES;            // a 128-row Q or K tile
    static constexpr int V_BYTES = kTileN * HD * 2;          // column blocks of 64 features
    static constexpr int NK = I8 ? 4 : (HD == 64 ? 6 : 3);   // (fp16: the 32 KB K tiles of 128-wide heads leave room
    static constexpr int NV = I8 ? 3 : (HD == 64 ? 4 : 2);   //  for fewer stages)
    static constexpr int KSTEPS = I8 ? 4 : HD / 16;          // MMAs per 64-key half of Q.K^T (K = 32 int8 / 16 fp16)
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + NQ * TILE_B;
    static constexpr int OFF_V = OFF_K + NK * TILE_B;
    static constexpr int OFF_BAR = OFF_V + NV * V_BYTES;
    // q_full, k_full[NK], k_empty[NK], v_full[NV], v_empty[NV], hi_full[2], lo_full[2], hi_free[2], p_full[2],
    // mma_done[2]
    static constexpr int NBAR = 1 + 2 * NK + 2 * NV + 10;
    static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr int SMEM = OFF_MISC + 16 + 1024;
    static constexpr int THREADS = 384;
    static constexpr uint32_t IDESC_QK = I8 ? idesc(kFmtS32, kFmtS8, kFmtS8, 0, 0, kTileM, 64)   // one half: N = 64 keys
                                            : idesc(kFmtF32, kFmtF16, kFmtF16, 0, 0, kTileM, 64);
    static constexpr uint32_t IDESC_PV = idesc(kFmtF32, kFmtF16, kFmtF16, 0, 1, kTileM, HD);
    static_assert(SMEM <= 232448, "shared memory budget of one sm_100 CTA");
    static_assert(8 * kStageWarpBytes <= OFF_V, "the output stage of the 8 softmax warps fits in Q and the K ring");
};

// One half row (64 keys) of scores r: keys at or past `valid` are masked. I8: r holds raw int32 sums; masked keys get
// kMaskedRaw, then the bias is added in place; returns the biased max. !I8: r holds fp32 scores; masked keys get -inf;
// returns the max.
template <bool I8>
__device__ __forceinline__ float sage3_bias_max(uint32_t (&r)[2][32], int valid) {
    if (valid < 64) {
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (c2 * 32 + i >= valid) r[c2][i] = I8 ? kMaskedRaw : 0xFF800000u;
    }
    if (I8) {
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
            for (int i = 0; i < 32; ++i) r[c2][i] += kBias;
    }
    return fmaxf(max32(r[0]), max32(r[1]));
}
// The exp argument's offset for running max m (log2 units) and scale c: I8 removes the bias too.
template <bool I8>
__device__ __forceinline__ float sage3_offset(float c, float m) {
    if (m == -INFINITY) return 0.0f;           // still no valid key: every weight is 0, not NaN
    return I8 ? -fmaf(kBiasF, c, m) : -m;
}
template <bool I8>
__device__ __forceinline__ float sage3_scaled_max(float bm, float c) {
    if (bm == -INFINITY) return -INFINITY;
    return I8 ? (bm - kBiasF) * c : bm * c;
}

// exp2 of one half row's 64 biased scores: p = 2^(r*c + k), rounded to half and packed two per word into pk; returns
// the sum of the p. FMAs and sums on packed f32x2 instructions.
__device__ __forceinline__ float sage3_exp_half(const uint32_t (&r)[2][32], float c, float k, uint32_t (&pk)[32]) {
    const float2 c2v = make_float2(c, c), k2v = make_float2(k, k);
    float2 sum[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const float2 y = __ffma2_rn(make_float2(__uint_as_float(r[c2][2 * e]), __uint_as_float(r[c2][2 * e + 1])), c2v, k2v);
            float2 p;
            p.x = ex2(y.x);
            p.y = ex2(y.y);
            sum[e & 3] = __fadd2_rn(sum[e & 3], p);
            pk[c2 * 16 + e] = pack_half2(p.x, p.y);
        }
    const float2 s01 = __fadd2_rn(sum[0], sum[1]), s23 = __fadd2_rn(sum[2], sum[3]);
    const float2 s = __fadd2_rn(s01, s23);
    return s.x + s.y;
}

template <bool I8, int HD = kHeadDim>
__global__ void __launch_bounds__(Sage3Cfg<I8, HD>::THREADS, 1)
    attn_sage3(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
    using C = Sage3Cfg<I8, HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
    uint64_t* q_full = bar;
    uint64_t* k_full = bar + 1;
    uint64_t* k_empty = k_full + C::NK;
    uint64_t* v_full = k_empty + C::NK;
    uint64_t* v_empty = v_full + C::NV;
    uint64_t* hi_full = v_empty + C::NV;   // [tile]: S_hi_t(j) complete
    uint64_t* lo_full = hi_full + 2;       // [tile]: S_lo_t(j) complete (and every earlier MMA); a last phase after the last P.V
    uint64_t* hi_free = lo_full + 2;       // [tile], one arrival per softmax warp: S_hi_t(j) read into registers
    uint64_t* p_full = hi_free + 2;        // [tile], one arrival per softmax warp: P_t(j) in TMEM, O_t rescaled
    uint64_t* mma_done = p_full + 2;       // [tile]: every MMA of that tile's issuer complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::OFF_MISC);
    volatile int* abort = reinterpret_cast<volatile int*>(sm + C::OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y % a.H, b = blockIdx.y / a.H;
    const int q0 = blockIdx.x * (C::NQ * kTileM);
    const int n_kv = a.n_kv;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        // a K or V stage is free once both MMA warps have committed their last use of it
        for (int i = 0; i < C::NK; ++i) { mbar_init(k_full + i, 1); mbar_init(k_empty + i, 2); }
        for (int i = 0; i < C::NV; ++i) { mbar_init(v_full + i, 1); mbar_init(v_empty + i, 2); }
        for (int t = 0; t < 2; ++t) {
            mbar_init(hi_full + t, 1);
            mbar_init(lo_full + t, 1);
            mbar_init(hi_free + t, 4);
            mbar_init(p_full + t, 4);
            mbar_init(mma_done + t, 1);
        }
        *abort = *reinterpret_cast<volatile int*>(a.err) != 0;   // a failed launch: no work in this CTA
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto fail = [&](int code) {
        atomicOr(a.err, code);
        *abort = 1;
    };
    const bool skip = *abort != 0;

    if (skip) {
    } else if (warp == 0 || warp == 2) {
        // ---------------- TMA producers: warp 0 loads Q and the K ring, warp 2 the V ring ----------------
        if (lane == 0) {
            const bool kq = warp == 0;
            bool ok = true;
            int last[C::NK > C::NV ? C::NK : C::NV];
            for (int i = 0; i < (C::NK > C::NV ? C::NK : C::NV); ++i) last[i] = -1;
            if (kq) {
                tma_prefetch_desc(&tmQ);
                tma_prefetch_desc(&tmK);
                mbar_expect_tx(q_full, C::NQ * C::TILE_B);
                for (int t = 0; t < C::NQ; ++t)
                    for (int cb = 0; cb < C::TILE_B / C::CB_BYTES; ++cb)
                        tma_rows(sm + C::OFF_Q + t * C::TILE_B + cb * C::CB_BYTES, &tmQ, q_full, a.q_order, cb * 64,
                                 q0 + t * kTileM, h, b);
            } else {
                tma_prefetch_desc(&tmV);
            }
            const int ns = kq ? C::NK : C::NV;
            uint64_t* full = kq ? k_full : v_full;
            uint64_t* empty = kq ? k_empty : v_empty;
            for (int j = 0; j < n_kv; ++j) {
                if (*reinterpret_cast<volatile int*>(a.err) != 0) { *abort = 1; ok = false; break; }
                const int st = j % ns;
                if (j >= ns && !mbar_wait(empty + st, ((j / ns) - 1) & 1, a.wait_ns, abort)) { ok = false; break; }
                if (kq) {
                    mbar_expect_tx(full + st, C::TILE_B);
                    for (int cb = 0; cb < C::TILE_B / C::CB_BYTES; ++cb)
                        tma_rows(sm + C::OFF_K + st * C::TILE_B + cb * C::CB_BYTES, &tmK, full + st, a.k_order, cb * 64,
                                 j * kTileN, h, b);
                } else {
                    mbar_expect_tx(full + st, C::V_BYTES);
                    for (int cb = 0; cb < HD / 64; ++cb)
                        tma_rows(sm + C::OFF_V + st * C::V_BYTES + cb * C::CB_BYTES, &tmV, full + st, a.v_order, cb * 64,
                                 j * kTileN, h, b);
                }
                last[st] = j;
            }
            if (!ok) fail(kErrProducer);
            // no copy may still be landing in shared memory when the CTA ends
            if (kq) mbar_wait(q_full, 0, a.wait_ns, nullptr);
            for (int i = 0; i < ns; ++i)
                if (last[i] >= 0) mbar_wait(full + i, (last[i] / ns) & 1, a.wait_ns, nullptr);
        }
        __syncwarp();
    } else if (warp == 1 || warp == 3) {
        // ---------------- MMA issuers: warp 1 for query tile 0, warp 3 for tile 1 (the whole warp runs the loop, one
        // elected lane issues). Two in-order streams, so that one tile's MMAs never queue behind a wait for the other
        // tile's softmax; each warp's commits track its own MMAs.
        const int t = warp == 1 ? 0 : 1;
        bool ok = warp_wait(q_full, 0, a.wait_ns, abort);
        // S_hi_t or S_lo_t = Q_t.K_j[half]^T (N = 64: rows 64*half.. of the K tile); K_j has landed
        auto qk = [&](int j, int half) {
            const int sk = j % C::NK;
            tc_fence_after();
            const uint32_t q_base = smem_u32(sm + C::OFF_Q + t * C::TILE_B);
            const uint32_t k_base = smem_u32(sm + C::OFF_K + sk * C::TILE_B + half * 64 * 128);
#pragma unroll
            for (int kk = 0; kk < C::KSTEPS; ++kk) {
                // 32 bytes of K per MMA; fp16 Q, K span two column blocks of 64 features
                const uint32_t off = (uint32_t) ((kk / 4) * C::CB_BYTES + (kk % 4) * 32);
                mma_ss_w<I8>(tmem + t * kTileN + half * 64, sdesc(q_base + off, 16, 1024), sdesc(k_base + off, 16, 1024),
                             C::IDESC_QK, kk > 0 ? 1u : 0u);
            }
        };
        // O_t += P_t(j).V_j; V_j has landed, P_t(j) is in TMEM
        auto pv = [&](int j) {
            const int sv = j % C::NV;
            tc_fence_after();
            const uint32_t v_base = smem_u32(sm + C::OFF_V + sv * C::V_BYTES);
#pragma unroll
            for (int kk = 0; kk < kTileN / 16; ++kk)
                mma_ts_f16_w(tmem + 2 * kTileN + t * HD, tmem + t * kTileN + kk * 8,
                             sdesc(v_base + (uint32_t) (kk * 16 * 128), C::CB_BYTES, 1024), C::IDESC_PV,
                             (j > 0 || kk > 0) ? 1u : 0u);
        };
        auto wait_k = [&](int j) { return warp_wait(k_full + j % C::NK, (j / C::NK) & 1, a.wait_ns, abort); };
        auto wait_v = [&](int j) { return warp_wait(v_full + j % C::NV, (j / C::NV) & 1, a.wait_ns, abort); };
        ok = ok && wait_k(0);
        if (ok) {
            qk(0, 1);
            mma_commit_w(hi_full + t);
            qk(0, 0);
            mma_commit_w(k_empty);
            mma_commit_w(lo_full + t);
        }
        for (int j = 0; j < n_kv && ok; ++j) {
            const bool more = j + 1 < n_kv;
            if (!wait_v(j) || (more && !wait_k(j + 1))) { ok = false; break; }
            // S_hi of the next key tile as soon as the softmax has read S_hi(j)
            if (more) {
                if (!warp_wait(hi_free + t, j & 1, a.wait_ns, abort)) { ok = false; break; }
                qk(j + 1, 1);
                mma_commit_w(hi_full + t);
            }
            if (!warp_wait(p_full + t, j & 1, a.wait_ns, abort)) { ok = false; break; }
            pv(j);
            mma_commit_w(v_empty + j % C::NV);
            if (more) {
                qk(j + 1, 0);
                mma_commit_w(k_empty + (j + 1) % C::NK);
            }
            // the next S_lo, or after the last P.V the phase the epilogue waits for
            mma_commit_w(lo_full + t);
        }
        if (!ok && lane == 0) fail(kErrMma);
        mma_commit_w(mma_done + t);
        mbar_wait(mma_done + t, 0, a.wait_ns, nullptr);
        __syncwarp();
    } else {
        // ---------------- softmax + epilogue: warps 4-7 tile 0, warps 8-11 tile 1 ----------------
        const int t = (warp - 4) >> 2;
        const int wq = warp & 3;                      // the TMEM lane quarter this warp may touch
        const int row = wq * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t) (wq * 32) << 16);
        const uint32_t colS = (uint32_t) (t * kTileN), colO = (uint32_t) (2 * kTileN + t * HD);
        const int qrow = q0 + t * kTileM + row;
        const int S = a.S;
        const float cq = I8 ? a.qs[(size_t) h * a.nb + min(qrow, S - 1) / a.blk] * a.scale_log2 : a.scale_log2;
        const float* ksh = a.ks + (size_t) h * a.nb;
        const int kpb = a.blk / 64;      // 64-key groups per scale block (1 for the reference's block of 64)
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        // the K scales of a tile are loaded one tile ahead
        auto ks_of = [&](int jj, float& lo, float& hi) {
            if (!I8) { lo = hi = 1.0f; return; }
            const int g = min(jj, n_kv - 1) * 2;
            lo = ksh[min(kpb == 1 ? g : g / kpb, a.nb - 1)];
            hi = ksh[min(kpb == 1 ? g + 1 : (g + 1) / kpb, a.nb - 1)];
        };
        float ks_lo, ks_hi;
        ks_of(0, ks_lo, ks_hi);
        // The warps of the two query tiles for this lane quarter share an SM sub-partition and its MUFU unit. They
        // take turns at the exps of each half tile (tile 0's, then tile 1's), so that one warp's loads, bias adds and
        // max trees run while the other's exps use the MUFU unit. The turns pass on two named barriers per quarter
        // (a hardware wait). Every warp makes the same sequence of 2 * n_kv turns on every path: after a failure it
        // takes the turns it has left without work, so the other warp is never left waiting.
        const uint32_t bar_to1 = 1 + 2 * wq, bar_to0 = 2 + 2 * wq;
        auto take_turn = [&](bool first) {
            if (t == 1) bar_sync(bar_to1, 64);
            else if (!first) bar_sync(bar_to0, 64);
        };
        auto give_turn = [&] { bar_arrive(t == 0 ? bar_to1 : bar_to0, 64); };
        int turns = 0;                     // turns taken and given back
        for (int j = 0; j < n_kv; ++j) {
            const int kv0 = j * kTileN;
            // c > 0 always (a zero scale gives zero scores either way), so -inf keys stay -inf through the FFMA
            const float c_lo = fmaxf(cq * ks_lo, 1e-30f);
            const float c_hi = fmaxf(cq * ks_hi, 1e-30f);
            // the next tile's scales load into the same registers: nothing waits for them before the next iteration
            ks_of(j + 1, ks_lo, ks_hi);
            const float m_prev = m_run;

            // ---- keys 64-127: read, free the columns for the next tile, max, exps (P_hi stays in registers)
            ok = warp_wait(hi_full + t, j & 1, a.wait_ns, abort);
            if (!ok) break;
            tc_fence_after();
            uint32_t r[2][32];
            tmem_ld32(t_lane + colS + 64, r[0]);
            tmem_ld32(t_lane + colS + 96, r[1]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(hi_free + t);
            const float bm_hi = sage3_bias_max<I8>(r, S - kv0 - 64);
            const float sm_hi = sage3_scaled_max<I8>(bm_hi, c_hi);
            if (sm_hi > m_run + 8.0f) m_run = sm_hi;             // also the first finite max
            const float m_hi = m_run;                             // the max the P_hi weights are taken against
            uint32_t p_hi[32];
            take_turn(turns == 0);
            float sum_hi = sage3_exp_half(r, c_hi, sage3_offset<I8>(c_hi, m_run), p_hi);
            give_turn();
            ++turns;

            // ---- keys 0-63: read (after P(j-1).V_{j-1}), max, and where the max moves, scale P_hi down
            ok = warp_wait(lo_full + t, j & 1, a.wait_ns, abort);
            if (!ok) break;
            tc_fence_after();
            tmem_ld32(t_lane + colS, r[0]);
            tmem_ld32(t_lane + colS + 32, r[1]);
            tmem_wait_ld();
            const float bm_lo = sage3_bias_max<I8>(r, S - kv0);
            const float sm_lo = sage3_scaled_max<I8>(bm_lo, c_lo);
            if (sm_lo > m_run + 8.0f) m_run = sm_lo;
            if (__any_sync(0xffffffffu, m_run != m_hi)) {
                // rare: the low keys moved the max past the one P_hi was taken against (or P_hi had no finite max)
                const float f = m_run == m_hi ? 1.0f : (m_hi == -INFINITY ? 0.0f : ex2(m_hi - m_run));
                const __half2 f2 = __float2half2_rn(f);
                sum_hi *= f;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    __half2 v = *reinterpret_cast<__half2*>(&p_hi[i]);
                    v = __hmul2(v, f2);
                    p_hi[i] = *reinterpret_cast<uint32_t*>(&v);
                }
            }
            uint32_t p_lo[32];
            // P_hi goes to TMEM columns 32-63 (S_lo's, read above). The fp16 kernel issues those stores inside its lo
            // turn, before the exps: measured 15-20 % shorter (32 heads x 8,192 tokens: 0.86-0.92 ms against
            // 1.08-1.12 ms). The int8 kernel is no faster that way and keeps them after the lo stores.
            auto store_p_hi = [&] {
                tmem_st16(t_lane + colS + 32, *reinterpret_cast<const uint32_t(*)[16]>(&p_hi[0]));
                tmem_st16(t_lane + colS + 48, *reinterpret_cast<const uint32_t(*)[16]>(&p_hi[16]));
            };
            take_turn(false);
            if constexpr (!I8) store_p_hi();
            const float sum_lo = sage3_exp_half(r, c_lo, sage3_offset<I8>(c_lo, m_run), p_lo);
            give_turn();
            ++turns;
            tmem_st16(t_lane + colS, *reinterpret_cast<const uint32_t(*)[16]>(&p_lo[0]));
            tmem_st16(t_lane + colS + 16, *reinterpret_cast<const uint32_t(*)[16]>(&p_lo[16]));
            if constexpr (I8) store_p_hi();
            // l and O: scaled by 2^(m_prev - m_run) where the max moved in this tile
            const bool grow = m_run != m_prev;
            const float alpha = grow ? (m_prev == -INFINITY ? 0.0f : ex2(m_prev - m_run)) : 1.0f;
            l_run = fmaf(l_run, alpha, sum_hi + sum_lo);
            // O_t holds the sum up to tile j-1 (S_lo(j) is complete)
            if (__any_sync(0xffffffffu, grow && j > 0)) {
                const float al = j > 0 ? alpha : 1.0f;
#pragma unroll
                for (int c4 = 0; c4 < HD / 32; ++c4) {
                    uint32_t o[32];
                    tmem_ld32(t_lane + colO + c4 * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * al);
                    tmem_st32(t_lane + colO + c4 * 32, o);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full + t);
        }
        // the turns this warp has left after a failure, without work (the failure is recorded first, so that the
        // other roles stop waiting at once)
        if (!ok && lane == 0) fail(kErrSoftmax);
        for (; turns < 2 * n_kv; ++turns) {
            take_turn(turns == 0);
            give_turn();
        }
        // tile 1's last hand-back is taken here, so that no named barrier is left half arrived
        if (t == 0 && n_kv > 0) bar_sync(bar_to0, 64);
        // the final P_t.V: the MMA thread commits lo_full once more after the last one
        if (ok) ok = warp_wait(lo_full + t, n_kv & 1, a.wait_ns, abort);
        if (!ok) {
            if (lane == 0) fail(kErrSoftmax);
        } else {
            tc_fence_after();
            // every Q.K^T MMA of both tiles is complete here (the other tile's last S_lo was read before this
            // warp's last turn or the hand-back above), so Q and the K ring are free to stage the output rows
            if (a.out_vec) store_out_staged(a, b, h, qrow - lane, lane, t_lane + colO, 1.0f / l_run,
                                            sm + C::OFF_Q + (warp - 4) * kStageWarpBytes);
            else store_out_row(a, b, h, qrow, t_lane + colO, 1.0f / l_run, qrow < S);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// grid (query-tile pairs, heads x sequences)
template <bool I8, int HD = kHeadDim>
inline cudaError_t launch_sage3(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const AttnArgs& a,
                                int B, cudaStream_t st) {
    using C = Sage3Cfg<I8, HD>;
    cudaError_t e = cudaFuncSetAttribute(attn_sage3<I8, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned) ((a.S + C::NQ * kTileM - 1) / (C::NQ * kTileM)), (unsigned) (a.H * B));
    attn_sage3<I8, HD><<<grid, C::THREADS, C::SMEM, st>>>(q, k, v, a);
    return cudaGetLastError();
}

// The Sage kernel behind every entry point.
inline cudaError_t launch_sage(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const AttnArgs& a,
                               cudaStream_t st) {
    return launch_sage3<true>(q, k, v, a, 1, st);
}
// The fp16 SDPA behind every entry point: the 64-wide form for heads up to 64 wide.
inline cudaError_t launch_sdpa(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const AttnArgs& a, int B,
                               cudaStream_t st) {
    return a.D <= 64 ? launch_sage3<false, 64>(q, k, v, a, B, st) : launch_sage3<false>(q, k, v, a, B, st);
}

}  // namespace h3
