// attn2.cuh - the SageAttention v1 core for sm_100a with two 128-row query tiles per CTA (256 query rows).
//
// The int8 Q.K^T of both tiles runs on tcgen05 kind::i8 (int32 in TMEM), P.V on kind::f16 with P read from TMEM (fp32
// accumulator in TMEM), so shared memory only feeds Q, K and V to the tensor core. Two softmax warpgroups, one per query
// tile, alternate naturally with the tensor core: while one works on its scores, the MMAs of the other tile run.
// 12 warps in three warpgroups:
//   warp 0      TMA producer of Q0, Q1 (once) and the ring of int8 K tiles of 128 keys (128-byte swizzle)
//   warp 1      TMEM owner and MMA issuer (the whole warp runs the loop with uniform operands; elect.sync picks the
//               lane that issues): per key tile j, in this order: O0 += P0(j).V_j, S0 = Q0.K_{j+1}^T,
//               O1 += P1(j).V_j, S1 = Q1.K_{j+1}^T
//   warp 2      TMA producer of the ring of half V tiles
//   warp 3      idle (the softmax warpgroups start at warp 4 so that warp w reads TMEM lane quarter w % 4)
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1: one thread per query row (TMEM lane = row)
// TMEM: S0 columns 0-127, S1 128-255, O0 256-383, O1 384-511; P_t(j) (half, two per column) overwrites columns 0-63 of
// S_t once the softmax has read S_t(j). S_t(j+1) overwrites P_t(j): the MMAs issued by one thread run in issue order, so
// O_t += P_t(j).V_j has read P_t(j) before S_t = Q_t.K_{j+1}^T writes there. A commit counts every MMA issued before it,
// so when S_t(j) is complete, O_t holds the sum up to tile j-1 and the softmax may rescale it.
//
// Softmax arithmetic per element (log2 units): the int32 dot product x becomes a float by adding the bits of 1.5*2^23
// (exact for |x| < 2^22; here |x| <= 128*127*127), and one FFMA applies the dequantisation scale qs*ks*scale*log2(e)
// and subtracts the running max: arg = (1.5*2^23 + x)*c - (1.5*2^23*c + m). Row maxima use three-input max trees over
// the biased values of each 64-key scale block. The running max moves only when it grows by more than 8 (2^8 in the
// weights), which keeps O rescaling rare; P is rounded to half.
#pragma once
#include "attn.cuh"

namespace h3 {

struct Sage2Cfg {
    static constexpr int NQ = 2;                             // query tiles per CTA
    static constexpr int TILE_B = 128 * 128;                 // a 128-row int8 Q or K tile: one 128-byte column block
    static constexpr int V_BYTES = kTileN * kHeadDim * 2;    // 32 KB, two column blocks of 64 features
    static constexpr int CB_BYTES = 128 * 128;
    static constexpr int NK = 4, NV = 3;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + NQ * TILE_B;
    static constexpr int OFF_V = OFF_K + NK * TILE_B;
    static constexpr int OFF_BAR = OFF_V + NV * V_BYTES;
    // q_full, k_full[NK], k_empty[NK], v_full[NV], v_empty[NV], s_full[2], p_full[2], mma_done
    static constexpr int NBAR = 1 + 2 * NK + 2 * NV + 5;
    static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr int SMEM = OFF_MISC + 16 + 1024;
    static constexpr int THREADS = 384;
    static constexpr uint32_t IDESC_QK = idesc(kFmtS32, kFmtS8, kFmtS8, 0, 0, kTileM, kTileN);
    static constexpr uint32_t IDESC_PV = idesc(kFmtF32, kFmtF16, kFmtF16, 0, 1, kTileM, kHeadDim);
    static_assert(SMEM <= 232448, "shared memory budget of one sm_100 CTA");
};

// Phase timestamps for kernel development (compiled out unless H3_TRACE is defined): lane 0 of the first warp of
// each softmax warpgroup and the MMA thread of CTA (0, 0) record clock64() into h3_trace[role][tile][event].
#ifdef H3_TRACE
__device__ unsigned long long h3_trace[16][64][8];
#define H3_T(role, j, ev)                                                                         \
    do {                                                                                          \
        if (blockIdx.x == 0 && blockIdx.y == 0 && (j) < 64) h3_trace[role][j][ev] = clock64();    \
    } while (0)
#else
#define H3_T(role, j, ev) \
    do {                  \
    } while (0)
#endif

constexpr uint32_t kBias = 0x4B400000u;          // the bits of 1.5 * 2^23
constexpr float kBiasF = 12582912.0f;

// 2^x on the FMA pipe, for a share of the exponentials taken off the MUFU unit (16 per clock per SM). Round-to-nearest
// split x = n + f with f in [-0.5, 0.5] (adding 1.5*2^23 puts n in the low bits), 2^f by a degree-3 polynomial fitted
// here in relative error (minimax, max relative error 7.5e-5 over the interval; P is rounded to half afterwards), and
// n added into the exponent field. x is clamped at -125 so that the exponent stays normal; such weights round to 0 in
// half anyway, and -inf (keys past S) gives 0 too.
__device__ __forceinline__ float exp2_poly(float x) {
    x = fmaxf(x, -125.0f);
    const float t = x + kBiasF;
    const float f = x - (t - kBiasF);
    float p = fmaf(0.0551716685f, f, 0.242611125f);
    p = fmaf(p, f, 0.693260968f);
    p = fmaf(p, f, 0.999928057f);
    return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));   // unsigned: wraps, no overflow
}

// Of every 4 key pairs, this many go through exp2_poly, the rest through ex2.approx (MUFU).
#ifndef H3_POLY_PAIRS
#define H3_POLY_PAIRS 0
#endif
constexpr int kPolyPairs = H3_POLY_PAIRS;

// 16 consecutive 32-bit columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// exp2 of one row's 128 scores (arg = s*c + k, fp32), rounded to half and stored two per column into TMEM columns
// p_taddr .. p_taddr+63 (the P operand of the next MMA), with the row's sum of them. Keys past S hold -inf and c > 0,
// so their weight is exactly 0.
__device__ __forceinline__ float sage_exp_row(const uint32_t (&r)[4][32], float c_lo, float k_lo, float c_hi, float k_hi,
                                              uint32_t p_taddr) {
    float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {              // 32 keys -> 16 columns of P
        uint32_t pk[16];
        const float cc = c4 < 2 ? c_lo : c_hi, kk = c4 < 2 ? k_lo : k_hi;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const float x0 = fmaf(__uint_as_float(r[c4][2 * e]), cc, kk);
            const float x1 = fmaf(__uint_as_float(r[c4][2 * e + 1]), cc, kk);
            float p0, p1;
            if ((e & 3) < 4 - kPolyPairs) {
                p0 = ex2(x0);
                p1 = ex2(x1);
            } else {
                p0 = exp2_poly(x0);
                p1 = exp2_poly(x1);
            }
            sum[(2 * e) & 7] += p0;
            sum[(2 * e + 1) & 7] += p1;
            pk[e] = pack_half2(p0, p1);
        }
        tmem_st16(p_taddr + c4 * 16, pk);
    }
    return ((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7]));
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
    uint64_t* s_full = v_empty + C::NV;    // [tile]: S_t(j) complete (and every earlier MMA)
    uint64_t* p_full = s_full + 2;         // [tile], 128 arrivals: P_t(j) in TMEM, O_t rescaled
    uint64_t* mma_done = p_full + 2;
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
            mbar_init(p_full + t, 128);
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

    if (skip || warp == 3) {
    } else if (warp == 0 || warp == 2) {
        // ---------------- TMA producers: warp 0 loads Q and the K ring, warp 2 the V ring ----------------
        // (separate threads, so that a K tile is never held up behind a V stage that is still in use)
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
                    tma_rows(sm + C::OFF_Q + t * C::TILE_B, &tmQ, q_full, a.q_order, 0, q0 + t * kTileM, h, b);
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
                    tma_rows(sm + C::OFF_K + st * C::TILE_B, &tmK, full + st, a.k_order, 0, j * kTileN, h, b);
                } else {
                    mbar_expect_tx(full + st, C::V_BYTES);
                    for (int cb = 0; cb < 2; ++cb)
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
    } else if (warp == 1) {
        // ---------------- MMA issuer: the whole warp runs it, one elected lane issues ----------------
        const unsigned all = 0xffffffffu;
        bool ok = __all_sync(all, mbar_wait(q_full, 0, a.wait_ns, abort));
        auto qk = [&](int t, int j) -> bool {
            const int sk = j % C::NK;
            if (t == 0 && !__all_sync(all, mbar_wait(k_full + sk, (j / C::NK) & 1, a.wait_ns, abort))) return false;
            tc_fence_after();
            const uint32_t q_base = smem_u32(sm + C::OFF_Q + t * C::TILE_B);
            const uint32_t k_base = smem_u32(sm + C::OFF_K + sk * C::TILE_B);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                mma_ss_w<true>(tmem + t * kTileN, sdesc(q_base + kk * 32, 16, 1024), sdesc(k_base + kk * 32, 16, 1024),
                               C::IDESC_QK, kk > 0 ? 1u : 0u);
            if (t == 1) mma_commit_w(k_empty + sk);
            mma_commit_w(s_full + t);
            return true;
        };
        auto pv = [&](int t, int j) -> bool {
            const int sv = j % C::NV;
            if (!__all_sync(all, mbar_wait(p_full + t, j & 1, a.wait_ns, abort))) return false;
            if (t == 0 && !__all_sync(all, mbar_wait(v_full + sv, (j / C::NV) & 1, a.wait_ns, abort))) return false;
            tc_fence_after();
            const uint32_t v_base = smem_u32(sm + C::OFF_V + sv * C::V_BYTES);
#pragma unroll
            for (int kk = 0; kk < kTileN / 16; ++kk)
                mma_ts_f16_w(tmem + 2 * kTileN + t * kHeadDim, tmem + t * kTileN + kk * 8,
                             sdesc(v_base + (uint32_t) (kk * 16 * 128), C::CB_BYTES, 1024), C::IDESC_PV,
                             (j > 0 || kk > 0) ? 1u : 0u);
            if (t == 1) mma_commit_w(v_empty + sv);
            return true;
        };
        ok = ok && qk(0, 0) && qk(1, 0);
        for (int j = 0; j < n_kv && ok; ++j) {
            if (lane == 0) H3_T(2, j, 0);
            if (!pv(0, j)) { ok = false; break; }
            if (lane == 0) H3_T(2, j, 1);
            if (j + 1 < n_kv && !qk(0, j + 1)) { ok = false; break; }
            if (lane == 0) H3_T(2, j, 2);
            if (!pv(1, j)) { ok = false; break; }
            if (lane == 0) H3_T(2, j, 3);
            if (j + 1 < n_kv && !qk(1, j + 1)) { ok = false; break; }
            if (lane == 0) H3_T(2, j, 4);
        }
        if (ok) {
            // after the last P.V of each tile: the epilogues wait for this phase of s_full
            mma_commit_w(s_full);
            mma_commit_w(s_full + 1);
        } else if (lane == 0) {
            fail(kErrMma);
        }
        mma_commit_w(mma_done);
        mbar_wait(mma_done, 0, a.wait_ns, nullptr);
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
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        const bool tr = (warp & 3) == 0 && lane == 0;
        // the K scales of a tile are loaded one tile ahead (a global load must not sit on the critical path)
        auto ks_of = [&](int jj, float& lo, float& hi) {
            const int k0 = min(jj, n_kv - 1) * kTileN;
            lo = ksh[min(k0 / a.blk, a.nb - 1)];
            hi = ksh[min((k0 + 64) / a.blk, a.nb - 1)];
        };
        float ks_lo, ks_hi;
        ks_of(0, ks_lo, ks_hi);
        for (int j = 0; j < n_kv; ++j) {
            float ks_lo_next, ks_hi_next;
            ks_of(j + 1, ks_lo_next, ks_hi_next);
            if (tr) H3_T(t, j, 0);
            // S_t(j) complete, and with it P_t(j-1).V: O_t is stable
            ok = __all_sync(0xffffffffu, mbar_wait(s_full + t, j & 1, a.wait_ns, abort));
            if (!ok) break;
            if (tr) H3_T(t, j, 1);
            tc_fence_after();
            uint32_t r[4][32];
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) tmem_ld32(t_lane + colS + c4 * 32, r[c4]);
            tmem_wait_ld();

            const int kv0 = j * kTileN;
            // int32 -> biased float (1.5*2^23 + x), keys past S excluded from the maxima
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
                for (int i = 0; i < 32; ++i) r[c4][i] += kBias;
            if (kv0 + kTileN > S) {
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (kv0 + c4 * 32 + i >= S) r[c4][i] = __float_as_uint(-INFINITY);
            }
            // c > 0 always (a zero scale gives zero scores either way), so -inf keys stay -inf through the FFMA
            const float c_lo = fmaxf(cq * ks_lo, 1e-30f);
            const float c_hi = fmaxf(cq * ks_hi, 1e-30f);
            ks_lo = ks_lo_next;
            ks_hi = ks_hi_next;
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
            if (tr) H3_T(t, j, 2);
            l_run += sage_exp_row(r, c_lo, k_lo, c_hi, k_hi, t_lane + colS);
            if (tr) H3_T(t, j, 3);
            // rescale O_t (the sum up to tile j-1) in place when this row's max grew
            if (__any_sync(0xffffffffu, grow && j > 0)) {
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
            }
            tmem_wait_st();
            if (tr) H3_T(t, j, 4);
            tc_fence_before();
            mbar_arrive(p_full + t);
            if (tr) H3_T(t, j, 5);
        }
        // the final P_t.V (the MMA thread commits s_full once more after the last one)
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(s_full + t, n_kv & 1, a.wait_ns, abort));
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
