// attn.cuh - the non-causal attention kernel for sm_100a, in two instantiations:
//
//   attn_fwd<true>   SageAttention v1 core: int8 Q.K^T on tcgen05 kind::i8 (int32 in TMEM), dequantised with the
//                    per-64-row scales of Q and K, online softmax, P in half, P.V on tcgen05 kind::f16 (fp32 in TMEM).
//                    Replaces the ARK kernel libh3sage.so calls (kernels/sage.cpp:51-52).
//   attn_fwd<false>  fp16 SDPA: Q.K^T on kind::f16 with fp32 scores, the same softmax and P.V.
//                    Replaces oneDNN's fused SDPA graph (kernels/h3sycl.cpp:1464-1500).
//
// One CTA = one head x 128 query rows, 6 warps, warp-specialised:
//   warp 0      TMA producer: Q once, then K and V tiles of 128 keys into rings of shared memory (128-byte swizzle).
//   warp 1      TMEM owner and MMA issuer (one thread): S[j&1] = Q.K_j^T into TMEM, then O += P_j.V_j into TMEM,
//               with Q.K_{j+1}^T issued before P_j.V_j so the tensor core works while the softmax runs.
//   warps 2-5   softmax: one thread per query row = one TMEM lane. Reads S_j, keeps the running max in log2 units
//               (rescaling O only when the max grows by more than 2^8), writes P_j in half to shared memory in the
//               UMMA K-major 128-byte-swizzled layout, and finally writes O / l through half to the output.
// TMEM: S0 columns 0-127, S1 128-255, O 256-383 (512 allocated).
//
// Q, K, V reach shared memory through 3-D TMA maps over (D, token, head) in either order, so the token-major rows of
// the engine (stride 3*H*D inside the qkv buffer) are read in place. Rows past S are zero-filled by TMA; keys past S
// are masked to -inf; query rows past S are not stored.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <string>

#include "ptx.cuh"

namespace h3 {

enum Dt : int { F32 = 0, F16 = 1, BF16 = 2 };

constexpr int kTileM = 128;   // query rows per CTA
constexpr int kTileN = 128;   // keys per K/V tile
constexpr int kHeadDim = 128;
constexpr int kAttnThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr int kColS0 = 0, kColO = 256;

// error word bits a kernel sets when one of its waits gave up
constexpr int kErrProducer = 1, kErrMma = 2, kErrSoftmax = 4, kErrPrepass = 8;

struct AttnArgs {
    int S;                      // tokens per sequence
    int H;                      // heads (grid.y = H * sequences)
    int n_kv;                   // key tiles, ceil(S / 128)
    float scale_log2;           // softmax scale * log2(e)
    const float* qs;            // int8 path: Q scales [H, nb], one per `blk` rows
    const float* ks;            // int8 path: K scales [H, nb]
    int nb, blk;
    void* out;                  // output element (b, s, h, d) at out + b*out_seq + s*out_tok + h*out_head + d
    long long out_seq, out_tok, out_head;
    int out_dt;                 // F16 / BF16 / F32; values go through half first (kernels/h3sycl.cpp:1769-1771)
    int out_vec;                // 16-byte stores allowed (alignment checked on the host)
    int q_order, k_order, v_order;   // 0: map dims (D, S, H, B); 1: map dims (D, H, S, B)
    int* err;                   // device error word
    unsigned long long wait_ns; // limit of every wait
    int D;                      // head size, 64 or 128: the kernels run 128 wide, and a 64-wide head reads as zeros in
                                // features 64-127 (TMA fills what lies outside the tensor with zeros), so those
                                // features of Q.K^T add nothing and those of P.V come out 0 and are not stored
    // Output rows spread over the ranks of a Ulysses group (out_rows > 0): token s goes to out_peer[s / out_rows], a
    // rank's token shard in its own or another GPU's memory (base already at this rank's head columns), at row
    // s % out_rows; out is then unused. out_rows = 0: every row to out.
    int out_rows;
    void* out_peer[8];
};

template <bool I8>
struct AttnCfg {
    static constexpr int QK_ES = I8 ? 1 : 2;
    static constexpr int ROW_B = kHeadDim * QK_ES;     // bytes per Q/K row: 128 or 256
    static constexpr int QK_CB = ROW_B / 128;           // 128-byte column blocks per Q/K row
    static constexpr int CB_BYTES = 128 * 128;          // one column block of a 128-row tile
    static constexpr int Q_BYTES = kTileM * ROW_B;
    static constexpr int K_BYTES = kTileN * ROW_B;
    static constexpr int V_BYTES = kTileN * kHeadDim * 2;
    static constexpr int P_BYTES = kTileM * kTileN * 2;
    static constexpr int NK = I8 ? 3 : 2;
    static constexpr int NV = 2;
    static constexpr int NP = I8 ? 2 : 1;
    static constexpr int QK_KSTEPS = I8 ? 4 : 8;        // one MMA eats 32 bytes of K: 32 int8 or 16 half
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + NK * K_BYTES;
    static constexpr int OFF_P = OFF_V + NV * V_BYTES;
    static constexpr int OFF_BAR = OFF_P + NP * P_BYTES;
    // q_full, k_full[NK], k_empty[NK], v_full[NV], v_empty[NV], s_full[2], s_free[2], p_full[2], pv_done[2], mma_done
    static constexpr int NBAR = 1 + 2 * NK + 2 * NV + 9;
    static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr int SMEM = OFF_MISC + 16 + 1024;   // + room to align the base to 1024 bytes
    static constexpr uint32_t IDESC_QK = I8 ? idesc(kFmtS32, kFmtS8, kFmtS8, 0, 0, kTileM, kTileN)
                                            : idesc(kFmtF32, kFmtF16, kFmtF16, 0, 0, kTileM, kTileN);
    static constexpr uint32_t IDESC_PV = idesc(kFmtF32, kFmtF16, kFmtF16, 0, 1, kTileM, kHeadDim);
    static_assert(SMEM <= 232448, "shared memory budget of one sm_100 CTA");
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void tma_rows(void* dst, const CUtensorMap* map, uint64_t* bar, int order, int c0, int row,
                                         int head, int seq) {
    if (order) tma_load_4d(dst, map, bar, c0, head, row, seq);
    else tma_load_4d(dst, map, bar, c0, row, head, seq);
}


// 32 consecutive output features of one row (fp32 values already divided by the row sum), rounded to half, then to
// out_dt (kernels/h3sycl.cpp:1769-1771), stored at out + e0 elements.
__device__ __forceinline__ void store_out32(const AttnArgs& a, void* out, long long e0, const float (&val)[32]) {
    __half hv[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) hv[i] = __float2half_rn(val[i]);
    if (a.out_dt == F16) {
        __half* dst = reinterpret_cast<__half*>(out) + e0;
        if (a.out_vec) {
#pragma unroll
            for (int v = 0; v < 4; ++v) reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(hv)[v];
        } else {
            for (int i = 0; i < 32; ++i) dst[i] = hv[i];
        }
    } else if (a.out_dt == BF16) {
        __nv_bfloat16 bv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) bv[i] = __float2bfloat16_rn(__half2float(hv[i]));
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out) + e0;
        if (a.out_vec) {
#pragma unroll
            for (int v = 0; v < 4; ++v) reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(bv)[v];
        } else {
            for (int i = 0; i < 32; ++i) dst[i] = bv[i];
        }
    } else {
        float fv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) fv[i] = __half2float(hv[i]);
        float* dst = reinterpret_cast<float*>(out) + e0;
        if (a.out_vec) {
#pragma unroll
            for (int v = 0; v < 8; ++v) reinterpret_cast<float4*>(dst)[v] = reinterpret_cast<const float4*>(fv)[v];
        } else {
            for (int i = 0; i < 32; ++i) dst[i] = fv[i];
        }
    }
}

// The epilogue of one query row: O (fp32, the first a.D of 128 TMEM columns from o_taddr) / l, stored at
// out + b*out_seq + qrow*out_tok + h*out_head. Warp-collective (TMEM loads): every lane calls it; rows past S
// (live = false) load but do not store.
__device__ __forceinline__ void store_out_row(const AttnArgs& a, int b, int h, int qrow, uint32_t o_taddr, float inv, bool live) {
    void* out = a.out;
    int row = qrow;
    if (a.out_rows > 0 && live) {
        const int p = qrow / a.out_rows;
        row = qrow - p * a.out_rows;
        out = a.out_peer[p & 7];
    }
    const long long base = (long long) b * a.out_seq + (long long) row * a.out_tok + (long long) h * a.out_head;
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
        if (c4 * 32 >= a.D) break;
        uint32_t o[32];
        tmem_ld32(o_taddr + c4 * 32, o);
        tmem_wait_ld();
        if (!live) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]) * inv;
        store_out32(a, out, base + c4 * 32, v);
    }
}

// max of 32 values with three-input max instructions (a tree: 16 instructions, depth 4)
__device__ __forceinline__ float max32(const uint32_t (&r)[32]) {
    float m[11];
#pragma unroll
    for (int i = 0; i < 10; ++i) m[i] = fmax3(__uint_as_float(r[3 * i]), __uint_as_float(r[3 * i + 1]), __uint_as_float(r[3 * i + 2]));
    m[10] = fmaxf(__uint_as_float(r[30]), __uint_as_float(r[31]));
    const float a0 = fmax3(m[0], m[1], m[2]), a1 = fmax3(m[3], m[4], m[5]), a2 = fmax3(m[6], m[7], m[8]);
    return fmax3(fmax3(a0, a1, a2), m[9], m[10]);
}

template <bool I8>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
             const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
    using C = AttnCfg<I8>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
    uint64_t* q_full = bar;
    uint64_t* k_full = bar + 1;
    uint64_t* k_empty = k_full + C::NK;
    uint64_t* v_full = k_empty + C::NK;
    uint64_t* v_empty = v_full + C::NV;
    uint64_t* s_full = v_empty + C::NV;
    uint64_t* s_free = s_full + 2;
    uint64_t* p_full = s_free + 2;
    uint64_t* pv_done = p_full + 2;
    uint64_t* mma_done = pv_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::OFF_MISC);
    volatile int* abort = reinterpret_cast<volatile int*>(sm + C::OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y % a.H, b = blockIdx.y / a.H;
    const int q0 = blockIdx.x * kTileM;
    const int n_kv = a.n_kv;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < C::NK; ++i) { mbar_init(k_full + i, 1); mbar_init(k_empty + i, 1); }
        for (int i = 0; i < C::NV; ++i) { mbar_init(v_full + i, 1); mbar_init(v_empty + i, 1); }
        for (int i = 0; i < 2; ++i) {
            mbar_init(s_full + i, 1);
            mbar_init(s_free + i, 128);
            mbar_init(p_full + i, 128);
            mbar_init(pv_done + i, 1);
        }
        mbar_init(mma_done, 1);
        // a CTA of a launch that has already failed does no work (its results are void anyway)
        *abort = *reinterpret_cast<volatile int*>(a.err) != 0;
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
        // nothing issued, nothing to wait for
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
            mbar_expect_tx(q_full, C::Q_BYTES);
            for (int cb = 0; cb < C::QK_CB; ++cb)
                tma_rows(sm + C::OFF_Q + cb * C::CB_BYTES, &tmQ, q_full, a.q_order, cb * (128 / C::QK_ES), q0, h, b);
            for (int j = 0; j < n_kv; ++j) {
                const int sk = j % C::NK;
                // another CTA's failure stops this one at the next tile
                if (*reinterpret_cast<volatile int*>(a.err) != 0) { *abort = 1; ok = false; break; }
                if (j >= C::NK && !mbar_wait(k_empty + sk, ((j / C::NK) - 1) & 1, a.wait_ns, abort)) { ok = false; break; }
                mbar_expect_tx(k_full + sk, C::K_BYTES);
                for (int cb = 0; cb < C::QK_CB; ++cb)
                    tma_rows(sm + C::OFF_K + sk * C::K_BYTES + cb * C::CB_BYTES, &tmK, k_full + sk, a.k_order,
                             cb * (128 / C::QK_ES), j * kTileN, h, b);
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
            // no copy may still be landing in shared memory when the CTA ends
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
            const uint32_t q_base = smem_u32(sm + C::OFF_Q);
            bool ok = mbar_wait(q_full, 0, a.wait_ns, abort);
            auto issue_qk = [&](int j) -> bool {
                const int sk = j % C::NK, sb = j & 1;
                if (!mbar_wait(k_full + sk, (j / C::NK) & 1, a.wait_ns, abort)) return false;
                if (j >= 2 && !mbar_wait(s_free + sb, ((j - 2) >> 1) & 1, a.wait_ns, abort)) return false;
                tc_fence_after();
                const uint32_t k_base = smem_u32(sm + C::OFF_K + sk * C::K_BYTES);
#pragma unroll
                for (int kk = 0; kk < C::QK_KSTEPS; ++kk) {
                    const uint32_t off = (uint32_t) ((kk >> 2) * C::CB_BYTES + (kk & 3) * 32);
                    mma_ss<I8>(tmem + kColS0 + sb * kTileN, sdesc(q_base + off, 16, 1024), sdesc(k_base + off, 16, 1024),
                               C::IDESC_QK, kk > 0 ? 1u : 0u);
                }
                mma_commit(k_empty + sk);
                mma_commit(s_full + sb);
                return true;
            };
            if (ok) ok = issue_qk(0);
            for (int j = 0; j < n_kv && ok; ++j) {
                if (j + 1 < n_kv && !issue_qk(j + 1)) { ok = false; break; }
                const int sv = j % C::NV, pb = j % C::NP;
                if (!mbar_wait(p_full + (j & 1), (j >> 1) & 1, a.wait_ns, abort)) { ok = false; break; }
                if (!mbar_wait(v_full + sv, (j / C::NV) & 1, a.wait_ns, abort)) { ok = false; break; }
                tc_fence_after();
                const uint32_t p_base = smem_u32(sm + C::OFF_P + pb * C::P_BYTES);
                const uint32_t v_base = smem_u32(sm + C::OFF_V + sv * C::V_BYTES);
#pragma unroll
                for (int kk = 0; kk < kTileN / 16; ++kk) {
                    // P: K-major, 16 keys = 32 bytes per step; V: MN-major, 16 keys = 16 rows of 128 bytes per step,
                    // the second 64 features one column block (LBO) further on
                    const uint64_t ad = sdesc(p_base + (uint32_t) ((kk >> 2) * C::CB_BYTES + (kk & 3) * 32), 16, 1024);
                    const uint64_t bd = sdesc(v_base + (uint32_t) (kk * 16 * 128), C::CB_BYTES, 1024);
                    mma_ss<false>(tmem + kColO, ad, bd, C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(v_empty + sv);
                mma_commit(pv_done + (j & 1));
            }
            if (!ok) fail(kErrMma);
            // every MMA this thread issued has completed before TMEM is released
            mma_commit(mma_done);
            mbar_wait(mma_done, 0, a.wait_ns, nullptr);
        }
        __syncwarp();
    } else {
        // ---------------- softmax + epilogue (warps 2-5) ----------------
        const int wq = warp & 3;                     // the TMEM lane quarter this warp may touch
        const int row = wq * 32 + lane;              // query row in the tile == TMEM lane
        const uint32_t t_lane = tmem + ((uint32_t) (wq * 32) << 16);
        const int qrow = q0 + row;
        const int S = a.S;
        float cq = a.scale_log2;
        if constexpr (I8) cq = a.qs[(size_t) h * a.nb + min(qrow, S - 1) / a.blk] * a.scale_log2;
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int sb = j & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(s_full + sb, (j >> 1) & 1, a.wait_ns, abort));
            if (!ok) break;
            tc_fence_after();
            uint32_t r[4][32];
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) tmem_ld32(t_lane + kColS0 + sb * kTileN + c4 * 32, r[c4]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_free + sb);

            // scores in log2 units
            float c_lo = cq, c_hi = cq;
            if constexpr (I8) {
                // every 64-key half of the tile lies inside one scale block (blk is a multiple of 64)
                const int b0 = min(j * kTileN / a.blk, a.nb - 1), b1 = min((j * kTileN + 64) / a.blk, a.nb - 1);
                c_lo = cq * a.ks[(size_t) h * a.nb + b0];
                c_hi = cq * a.ks[(size_t) h * a.nb + b1];
            }
            const int kv0 = j * kTileN;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float f;
                    if constexpr (I8) f = (float) (int) r[c4][i] * (c4 < 2 ? c_lo : c_hi);
                    else f = __uint_as_float(r[c4][i]) * cq;
                    r[c4][i] = __float_as_uint(f);
                }
            if (kv0 + kTileN > S) {                  // the last tile: keys past S do not count
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (kv0 + c4 * 32 + i >= S) r[c4][i] = __float_as_uint(-INFINITY);
            }
            const float mt = fmax3(max32(r[0]), max32(r[1]), fmaxf(max32(r[2]), max32(r[3])));
            const float m_new = fmaxf(m_run, mt);
            const bool grow = m_new > m_run + 8.0f;  // first tile: m_run = -inf
            float alpha = 1.0f;
            if (grow) {
                alpha = ex2(m_run - m_new);
                l_run *= alpha;
                m_run = m_new;
            }
            // the P buffer is free once P_{j-NP}.V has completed
            if (j >= C::NP) {
                ok = __all_sync(0xffffffffu, mbar_wait(pv_done + ((j - C::NP) & 1), ((j - C::NP) >> 1) & 1, a.wait_ns, abort));
                if (!ok) break;
            }
            uint8_t* pt = sm + C::OFF_P + (j % C::NP) * C::P_BYTES;
            float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 16; ++c) {          // 16-byte chunks of 8 keys
                uint32_t pk[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i = c * 8 + 2 * e;
                    const float p0 = ex2(__uint_as_float(r[i >> 5][i & 31]) - m_run);
                    const float p1 = ex2(__uint_as_float(r[(i + 1) >> 5][(i + 1) & 31]) - m_run);
                    sum[2 * e] += p0;
                    sum[2 * e + 1] += p1;
                    pk[e] = pack_half2(p0, p1);
                }
                const int cb = c >> 3, ch = c & 7;
                uint4* dst = reinterpret_cast<uint4*>(pt + cb * C::CB_BYTES + row * 128 + ((ch ^ (row & 7)) << 4));
                *dst = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            l_run += ((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7]));
            // rescale O (which holds the sum up to tile j-1) in place when this row's max grew
            if (__any_sync(0xffffffffu, grow && j > 0)) {
                if (C::NP != 1) {
                    ok = __all_sync(0xffffffffu, mbar_wait(pv_done + ((j - 1) & 1), ((j - 1) >> 1) & 1, a.wait_ns, abort));
                    if (!ok) break;
                }
                tc_fence_after();
                const float al = (grow && j > 0) ? alpha : 1.0f;
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
                    uint32_t o[32];
                    tmem_ld32(t_lane + kColO + c4 * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * al);
                    tmem_st32(t_lane + kColO + c4 * 32, o);
                }
                tmem_wait_st();
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(p_full + (j & 1));
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done + ((n_kv - 1) & 1), ((n_kv - 1) >> 1) & 1, a.wait_ns, abort));
        if (!ok) {
            if (lane == 0) fail(kErrSoftmax);
        } else {
            tc_fence_after();
            store_out_row(a, b, h, qrow, t_lane + kColO, 1.0f / l_run, qrow < S);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---- host side ---------------------------------------------------------------------------------------------------------

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// A 4-D map of 128-row boxes over B sequences of a tensor with D features per (token, head). Strides in bytes.
// order 0: dims (D, S, H, B) (packed [B, H, S, D]); order 1: dims (D, H, S, B) (token-major rows: the head stride is the
// smaller one). Returns an empty string, or why the map cannot be made (TMA wants a 16-byte aligned base and strides).
inline std::string make_rows_map(CUtensorMap* m, const void* base, bool int8, int64_t D, int64_t S, int64_t H, int64_t B,
                                 int64_t tok_bytes, int64_t head_bytes, int64_t seq_bytes, int order) {
    auto enc = tensor_map_encoder();
    if (!enc) return "cuTensorMapEncodeTiled is not available from the driver";
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (tok_bytes & 15) || (head_bytes & 15) || (seq_bytes & 15))
        return "not 16-byte aligned";
    const int es = int8 ? 1 : 2;
    cuuint64_t dims[4];
    cuuint64_t strides[3];
    cuuint32_t box[4];
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    dims[0] = (cuuint64_t) D;
    dims[3] = (cuuint64_t) B;
    strides[2] = (cuuint64_t) (B > 1 ? seq_bytes : (order == 0 ? head_bytes * H : tok_bytes * S));
    box[0] = (cuuint32_t) (128 / es);
    box[3] = 1;
    if (order == 0) {
        dims[1] = (cuuint64_t) S; dims[2] = (cuuint64_t) H;
        strides[0] = (cuuint64_t) tok_bytes; strides[1] = (cuuint64_t) head_bytes;
        box[1] = 128; box[2] = 1;
    } else {
        dims[1] = (cuuint64_t) H; dims[2] = (cuuint64_t) S;
        strides[0] = (cuuint64_t) head_bytes; strides[1] = (cuuint64_t) tok_bytes;
        box[1] = 1; box[2] = 128;
    }
    const CUresult r = enc(m, int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                           const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return "cuTensorMapEncodeTiled failed (" + std::to_string((int) r) + ")";
    return {};
}

template <bool I8>
inline cudaError_t launch_attn(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const AttnArgs& a, int B,
                               cudaStream_t st) {
    using C = AttnCfg<I8>;
    cudaError_t e = cudaFuncSetAttribute(attn_fwd<I8>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned) ((a.S + kTileM - 1) / kTileM), (unsigned) (a.H * B));
    attn_fwd<I8><<<grid, kAttnThreads, C::SMEM, st>>>(q, k, v, a);
    return cudaGetLastError();
}

}  // namespace h3
