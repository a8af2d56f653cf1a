// attn2.cuh - the SageAttention v1 core for sm_100a with two 128-row query tiles per CTA (256 query rows).
//
// The int8 Q.K^T of both tiles runs on tcgen05 kind::i8 (int32 in TMEM), P.V on kind::f16 (fp32 in TMEM). Two softmax
// warpgroups, one per query tile, work on the two tiles' scores in turn while the tensor core works on the other tile,
// so every SM sub-partition has two softmax warps to interleave. 12 warps in three warpgroups:
//   warp 0      TMA producer: Q0, Q1 once; K (int8) and V (half) tiles of 128 keys into rings (128-byte swizzle)
//   warp 1      TMEM owner and MMA issuer: per key tile j, S0 = Q0.K_j^T, O0 += P0.V_j, S1 = Q1.K_j^T, O1 += P1.V_j, with
//               each S_t(j+1) issued as soon as softmax t has read S_t(j)
//   warps 2-3   idle (the softmax warpgroups start at warp 4 so that warp w reads TMEM lane quarter w % 4)
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1: one thread per query row (TMEM lane = row)
// 168 registers per thread (the per-sub-partition limit at 12 warps), no spills.
// TMEM: S0 columns 0-127, S1 128-255, O0 256-383, O1 384-511.
//
// Softmax arithmetic per element (log2 units): the int32 dot product x becomes a float by adding the bits of 1.5*2^23
// (exact for |x| < 2^22; here |x| <= 128*127*127), and one FFMA applies the dequantisation scale qs*ks*scale*log2(e)
// and subtracts the running max: arg = (1.5*2^23 + x)*c - (1.5*2^23*c + m). Row maxima use three-input max trees over
// the biased values of each 64-key scale block. The running max moves only when it grows by more than 8 (2^8 in the
// weights), which keeps O rescaling rare; P is rounded to half and written to shared memory in the UMMA layout.
#pragma once
#include "attn.cuh"

namespace h3 {

struct Sage2Cfg {
    static constexpr int NQ = 2;                             // query tiles per CTA
    static constexpr int TILE_B = 128 * 128;                 // a 128-row int8 Q or K tile: one 128-byte column block
    static constexpr int V_BYTES = kTileN * kHeadDim * 2;    // 32 KB, two column blocks of 64 features
    static constexpr int P_BYTES = kTileM * kTileN * 2;      // 32 KB, two column blocks of 64 keys
    static constexpr int CB_BYTES = 128 * 128;
    static constexpr int NK = 3, NV = 2;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + NQ * TILE_B;
    static constexpr int OFF_V = OFF_K + NK * TILE_B;
    static constexpr int OFF_P = OFF_V + NV * V_BYTES;
    static constexpr int OFF_BAR = OFF_P + NQ * P_BYTES;
    // q_full, k_full[NK], k_empty[NK], v_full[NV], v_empty[NV], s_full[2], s_free[2], p_full[2], pv_done[2], mma_done
    static constexpr int NBAR = 1 + 2 * NK + 2 * NV + 9;
    static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr int SMEM = OFF_MISC + 16 + 1024;
    static constexpr int THREADS = 384;
    static constexpr int REGS_LOW = 96, REGS_HIGH = 200;
    static_assert(128 * REGS_LOW + 256 * REGS_HIGH <= THREADS * 168, "register re-split above the launch's registers");
    static constexpr uint32_t IDESC_QK = idesc(kFmtS32, kFmtS8, kFmtS8, 0, 0, kTileM, kTileN);
    static constexpr uint32_t IDESC_PV = idesc(kFmtF32, kFmtF16, kFmtF16, 0, 1, kTileM, kHeadDim);
    static_assert(SMEM <= 232448, "shared memory budget of one sm_100 CTA");
};

constexpr uint32_t kBias = 0x4B400000u;          // the bits of 1.5 * 2^23
constexpr float kBiasF = 12582912.0f;

template <bool TAIL>
__device__ __forceinline__ void sage_exp_row(uint32_t (&r)[4][32], float c_lo, float k_lo, float c_hi, float k_hi, int kv0,
                                             int S, int row, uint8_t* pt, float (&sum)[8]) {
#pragma unroll
    for (int c = 0; c < 16; ++c) {                // 16-byte chunks of 8 keys
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i = c * 8 + 2 * e;
            const float cc = i < 64 ? c_lo : c_hi, kk = i < 64 ? k_lo : k_hi;
            float x0 = fmaf(__uint_as_float(r[i >> 5][i & 31]), cc, kk);
            float x1 = fmaf(__uint_as_float(r[(i + 1) >> 5][(i + 1) & 31]), cc, kk);
            if (TAIL) {
                if (kv0 + i >= S) x0 = -INFINITY;
                if (kv0 + i + 1 >= S) x1 = -INFINITY;
            }
            const float p0 = ex2(x0), p1 = ex2(x1);
            sum[2 * e] += p0;
            sum[2 * e + 1] += p1;
            pk[e] = pack_half2(p0, p1);
        }
        const int cb = c >> 3, ch = c & 7;
        uint4* dst = reinterpret_cast<uint4*>(pt + cb * Sage2Cfg::CB_BYTES + row * 128 + ((ch ^ (row & 7)) << 4));
        *dst = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
}

__global__ void __launch_bounds__(Sage2Cfg::THREADS, 1)
    attn_sage2(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
    using C = Sage2Cfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
    uint64_t* q_full = bar;
    uint64_t* k_full = bar + 1;
    uint64_t* k_empty = k_full + C::NK;
    uint64_t* v_full = k_empty + C::NK;
    uint64_t* v_empty = v_full + C::NV;
    uint64_t* s_full = v_empty + C::NV;    // [tile]
    uint64_t* s_free = s_full + 2;         // [tile], 128 arrivals
    uint64_t* p_full = s_free + 2;         // [tile], 128 arrivals
    uint64_t* pv_done = p_full + 2;        // [tile]
    uint64_t* mma_done = pv_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::OFF_MISC);
    volatile int* abort = reinterpret_cast<volatile int*>(sm + C::OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y % a.H, b = blockIdx.y / a.H;
    const int q0 = blockIdx.x * (C::NQ * kTileM);
    const int n_kv = a.n_kv;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < C::NK; ++i) { mbar_init(k_full + i, 1); mbar_init(k_empty + i, 1); }
        for (int i = 0; i < C::NV; ++i) { mbar_init(v_full + i, 1); mbar_init(v_empty + i, 1); }
        for (int t = 0; t < 2; ++t) {
            mbar_init(s_full + t, 1);
            mbar_init(s_free + t, 128);
            mbar_init(p_full + t, 128);
            mbar_init(pv_done + t, 1);
        }
        mbar_init(mma_done, 1);
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

    if (skip || warp == 2 || warp == 3) {
    } else if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            bool ok = true;
            int last_k[C::NK], last_v[C::NV];
            for (int i = 0; i < C::NK; ++i) last_k[i] = -1;
            for (int i = 0; i < C::NV; ++i) last_v[i] = -1;
            mbar_expect_tx(q_full, C::NQ * C::TILE_B);
            for (int t = 0; t < C::NQ; ++t)
                tma_rows(sm + C::OFF_Q + t * C::TILE_B, &tmQ, q_full, a.q_order, 0, q0 + t * kTileM, h, b);
            for (int j = 0; j < n_kv; ++j) {
                if (*reinterpret_cast<volatile int*>(a.err) != 0) { *abort = 1; ok = false; break; }
                const int sk = j % C::NK;
                if (j >= C::NK && !mbar_wait(k_empty + sk, ((j / C::NK) - 1) & 1, a.wait_ns, abort)) { ok = false; break; }
                mbar_expect_tx(k_full + sk, C::TILE_B);
                tma_rows(sm + C::OFF_K + sk * C::TILE_B, &tmK, k_full + sk, a.k_order, 0, j * kTileN, h, b);
                last_k[sk] = j;
                const int sv = j % C::NV;
                if (j >= C::NV && !mbar_wait(v_empty + sv, ((j / C::NV) - 1) & 1, a.wait_ns, abort)) { ok = false; break; }
                mbar_expect_tx(v_full + sv, C::V_BYTES);
                for (int cb = 0; cb < 2; ++cb)
                    tma_rows(sm + C::OFF_V + sv * C::V_BYTES + cb * C::CB_BYTES, &tmV, v_full + sv, a.v_order, cb * 64,
                             j * kTileN, h, b);
                last_v[sv] = j;
            }
            if (!ok) fail(kErrProducer);
            mbar_wait(q_full, 0, a.wait_ns, nullptr);
            for (int i = 0; i < C::NK; ++i)
                if (last_k[i] >= 0) mbar_wait(k_full + i, (last_k[i] / C::NK) & 1, a.wait_ns, nullptr);
            for (int i = 0; i < C::NV; ++i)
                if (last_v[i] >= 0) mbar_wait(v_full + i, (last_v[i] / C::NV) & 1, a.wait_ns, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = mbar_wait(q_full, 0, a.wait_ns, abort);
            auto qk = [&](int t, int j) -> bool {
                const int sk = j % C::NK;
                if (t == 0 && !mbar_wait(k_full + sk, (j / C::NK) & 1, a.wait_ns, abort)) return false;
                if (j > 0 && !mbar_wait(s_free + t, (j - 1) & 1, a.wait_ns, abort)) return false;
                tc_fence_after();
                const uint32_t q_base = smem_u32(sm + C::OFF_Q + t * C::TILE_B);
                const uint32_t k_base = smem_u32(sm + C::OFF_K + sk * C::TILE_B);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_ss<true>(tmem + t * kTileN, sdesc(q_base + kk * 32, 16, 1024), sdesc(k_base + kk * 32, 16, 1024),
                                 C::IDESC_QK, kk > 0 ? 1u : 0u);
                if (t == 1) mma_commit(k_empty + sk);
                mma_commit(s_full + t);
                return true;
            };
            auto pv = [&](int t, int j) -> bool {
                const int sv = j % C::NV;
                if (!mbar_wait(p_full + t, j & 1, a.wait_ns, abort)) return false;
                if (t == 0 && !mbar_wait(v_full + sv, (j / C::NV) & 1, a.wait_ns, abort)) return false;
                tc_fence_after();
                const uint32_t p_base = smem_u32(sm + C::OFF_P + t * C::P_BYTES);
                const uint32_t v_base = smem_u32(sm + C::OFF_V + sv * C::V_BYTES);
#pragma unroll
                for (int kk = 0; kk < kTileN / 16; ++kk) {
                    const uint64_t ad = sdesc(p_base + (uint32_t) ((kk >> 2) * C::CB_BYTES + (kk & 3) * 32), 16, 1024);
                    const uint64_t bd = sdesc(v_base + (uint32_t) (kk * 16 * 128), C::CB_BYTES, 1024);
                    mma_ss<false>(tmem + 2 * kTileN + t * kHeadDim, ad, bd, C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
                }
                if (t == 1) mma_commit(v_empty + sv);
                mma_commit(pv_done + t);
                return true;
            };
            ok = ok && qk(0, 0) && qk(1, 0);
            for (int j = 0; j < n_kv && ok; ++j) {
                if (j + 1 < n_kv && !qk(0, j + 1)) { ok = false; break; }
                if (!pv(0, j)) { ok = false; break; }
                if (j + 1 < n_kv && !qk(1, j + 1)) { ok = false; break; }
                if (!pv(1, j)) { ok = false; break; }
            }
            if (!ok) fail(kErrMma);
            mma_commit(mma_done);
            mbar_wait(mma_done, 0, a.wait_ns, nullptr);
        }
        __syncwarp();
    } else {
        // ---------------- softmax + epilogue: warps 4-7 tile 0, warps 8-11 tile 1 ----------------
        const int t = (warp - 4) >> 2;
        const int wq = warp & 3;                      // the TMEM lane quarter this warp may touch
        const int row = wq * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t) (wq * 32) << 16);
        const uint32_t colS = (uint32_t) (t * kTileN), colO = (uint32_t) (2 * kTileN + t * kHeadDim);
        const int qrow = q0 + t * kTileM + row;
        const int S = a.S;
        const float cq = a.qs[(size_t) h * a.nb + min(qrow, S - 1) / a.blk] * a.scale_log2;
        const float* ksh = a.ks + (size_t) h * a.nb;
        uint8_t* pt = sm + C::OFF_P + t * C::P_BYTES;
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            ok = __all_sync(0xffffffffu, mbar_wait(s_full + t, j & 1, a.wait_ns, abort));
            if (!ok) break;
            tc_fence_after();
            uint32_t r[4][32];
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) tmem_ld32(t_lane + colS + c4 * 32, r[c4]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_free + t);

            const int kv0 = j * kTileN;
            const bool tail = kv0 + kTileN > S;
            // int32 -> biased float (1.5*2^23 + x), keys past S excluded from the maxima
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
                for (int i = 0; i < 32; ++i) r[c4][i] += kBias;
            if (tail) {
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (kv0 + c4 * 32 + i >= S) r[c4][i] = __float_as_uint(-INFINITY);
            }
            const float c_lo = cq * ksh[min(kv0 / a.blk, a.nb - 1)];
            const float c_hi = cq * ksh[min((kv0 + 64) / a.blk, a.nb - 1)];
            const float bm_lo = fmaxf(max32(r[0]), max32(r[1])), bm_hi = fmaxf(max32(r[2]), max32(r[3]));
            const float sm_lo = bm_lo == -INFINITY ? -INFINITY : (bm_lo - kBiasF) * c_lo;
            const float sm_hi = bm_hi == -INFINITY ? -INFINITY : (bm_hi - kBiasF) * c_hi;
            const float m_new = fmax3(m_run, sm_lo, sm_hi);
            const bool grow = m_new > m_run + 8.0f;       // first tile: m_run = -inf
            float alpha = 1.0f;
            if (grow) {
                alpha = ex2(m_run - m_new);
                l_run *= alpha;
                m_run = m_new;
            }
            const float k_lo = -fmaf(kBiasF, c_lo, m_run), k_hi = -fmaf(kBiasF, c_hi, m_run);
            // P_t and O_t are free once P_t(j-1).V has completed
            if (j > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(pv_done + t, (j - 1) & 1, a.wait_ns, abort));
                if (!ok) break;
            }
            float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (tail) sage_exp_row<true>(r, c_lo, k_lo, c_hi, k_hi, kv0, S, row, pt, sum);
            else sage_exp_row<false>(r, c_lo, k_lo, c_hi, k_hi, kv0, S, row, pt, sum);
            l_run += ((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7]));
            if (__any_sync(0xffffffffu, grow && j > 0)) {
                tc_fence_after();
                const float al = (grow && j > 0) ? alpha : 1.0f;
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
                    uint32_t o[32];
                    tmem_ld32(t_lane + colO + c4 * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * al);
                    tmem_st32(t_lane + colO + c4 * 32, o);
                }
                tmem_wait_st();
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(p_full + t);
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done + t, (n_kv - 1) & 1, a.wait_ns, abort));
        if (!ok) {
            if (lane == 0) fail(kErrSoftmax);
        } else {
            tc_fence_after();
            store_out_row(a, b, h, qrow, t_lane + colO, 1.0f / l_run, qrow < S);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

inline cudaError_t launch_sage2(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const AttnArgs& a,
                                cudaStream_t st) {
    using C = Sage2Cfg;
    cudaError_t e = cudaFuncSetAttribute(attn_sage2, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned) ((a.S + C::NQ * kTileM - 1) / (C::NQ * kTileM)), (unsigned) a.H);
    attn_sage2<<<grid, C::THREADS, C::SMEM, st>>>(q, k, v, a);
    return cudaGetLastError();
}

}  // namespace h3
