// int8lin.cuh - the int8 "ConvRot" linear layer for sm_100a (kernels/h3sycl.h:74-85, kernels/h3sycl.cpp:404-652 of
// the reference):
//
//   x_rot = x . H          per group of g features, H the normalised Hadamard matrix h4 (x) h4 (x) ... (one h4 factor
//                          per base-4 digit of the feature index)
//   s_r   = max(max|x_rot[r]| / 127, 1e-30)                          per row
//   q     = clamp(rint(x_rot / s_r), -128, 127)                      int8
//   acc   = q . W^T                                                  int32, on the tensor cores
//   out   = acc * (s_r * ws)   (one weight scale)   or   (acc * s_r) * ws[n]   (one per output),   + bias[n]
//
// Two kernels:
//   rotq_rows  HBM-bound; one CTA per row at a time. A thread loads 16 consecutive features (16-byte loads) and applies
//              the two low digits of the rotation in its registers, in the order of the reference's fused kernel
//              (t = ((x_0 + x_1) + x_2) + x_3, y_c = t - 2 x_(3-c)). For groups of 32 and more the window goes through
//              shared memory once, so that each thread then holds the 2-16 values that differ only in the higher digits
//              (which the reference combines by lane shuffles, t = (x_0 + x_1) + (x_2 + x_3)): two shared-memory passes
//              in place of three shuffles per value and digit. A row of up to 16384 features stays in shared memory
//              between its absmax and its quantisation; a longer one is rotated twice (the same arithmetic, the same
//              bits).
//   i8gemm     persistent, one CTA per SM: 128 x 256 output tiles; a 4-stage TMA ring of 128-byte K slices (16 KB of
//              x_q and 32 KB of W per stage, 128-byte swizzle); tcgen05.mma kind::i8 into one of two 256-column int32
//              accumulators in tensor memory, so that the epilogue of one tile runs under the MMAs of the next.
//              Warp 0 loads, warp 1 issues the MMAs (one elected lane), warps 2-5 each read a quarter of the 128 lanes
//              (rows) and apply the rescale and the bias, one output row per thread.
//
// The rescale is the reference's post-op order (kernels/h3sycl.cpp:573-599): the single weight scale is folded into the
// row scale first (rs * ws); a per-output scale multiplies after the row scale; the bias comes last; every step is a
// round-to-nearest float32 operation (the _rn intrinsics, never contracted) and the result is rounded to the output
// type once.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "prepass.cuh"
#include "ptx.cuh"

namespace h3 {

// ---- rotation + quantisation ----------------------------------------------------------------------------------------
constexpr int kRqThreads = 256;
constexpr int kRqWin = 16 * kRqThreads;                              // features per window: 16 per thread
constexpr int kRqWinPad = kRqWin + kRqWin / 32 * 4 + kRqWin / 256 * 16;   // padded floats per window (4864)
constexpr int kRqResident = 4 * kRqWin;                              // rows up to this long stay in shared memory

// Shared-memory index of feature f of a row: 4 floats of padding per 32 and 16 more per 256 keep both the chunk
// stores (16 consecutive floats per thread, as float4) and the line reads of the high digits (16 lanes on 16
// consecutive floats, the next 16 lanes one group further) free of bank conflicts.
__device__ __forceinline__ int rq_pad(int f) { return f + (f >> 5) * 4 + (f >> 8) * 16; }

// base-4 digits of a group of G features (the reference's matrix builder halves the norm once per digit,
// kernels/h3sycl.cpp:189-190): 1/2 per digit
template <int G> struct RqDigits {
    static constexpr int N = G <= 1 ? 0 : G <= 4 ? 1 : G <= 16 ? 2 : G <= 64 ? 3 : 4;
    static constexpr float NORM = N == 0 ? 1.0f : N == 1 ? 0.5f : N == 2 ? 0.25f : N == 3 ? 0.125f : 0.0625f;
};

// One h4 digit of stride D over an array of NV values in groups of GS: for the four values v[e0 + c*D] of each
// digit, a sequential sum (inside a thread, the low digits) or a pairwise one (the high digits), then y_c = t - 2 x_(3-c)
// as one fma (2x is exact, so fma(-2, x, t) rounds t - 2x once, as the subtraction does). A digit with only two values
// (GS = 2 * D, the top digit of g = 2 * 4^n, where the reference's matrix has h4's corner [[1, 1], [1, 1]]): both
// become x_0 + x_1.
template <int NV, int GS, int D, bool SEQ>
__device__ __forceinline__ void rq_digit(float* v) {
    if constexpr (4 * D <= GS) {
#pragma unroll
        for (int e0 = 0; e0 < NV; ++e0) {
            if ((e0 / D) % 4 != 0) continue;
            const float a0 = v[e0], a1 = v[e0 + D], a2 = v[e0 + 2 * D], a3 = v[e0 + 3 * D];
            const float t = SEQ ? __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3) : __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
            v[e0] = __fmaf_rn(-2.0f, a3, t);
            v[e0 + D] = __fmaf_rn(-2.0f, a2, t);
            v[e0 + 2 * D] = __fmaf_rn(-2.0f, a1, t);
            v[e0 + 3 * D] = __fmaf_rn(-2.0f, a0, t);
        }
    } else {
#pragma unroll
        for (int e0 = 0; e0 < NV; ++e0) {
            if ((e0 / D) % 2 != 0) continue;
            const float s = __fadd_rn(v[e0], v[e0 + D]);
            v[e0] = s;
            v[e0 + D] = s;
        }
    }
}

// the digits of strides 1 and 4 inside a thread's 16 consecutive features (those below the group size)
template <int G>
__device__ __forceinline__ void rq_low(float (&v)[16]) {
    constexpr int GS = G < 16 ? G : 16;
    if constexpr (G > 1) rq_digit<16, GS, 1, true>(v);
    if constexpr (G > 4) rq_digit<16, GS, 4, true>(v);
}
// the digits of strides 1 and 4 over the G/16 values of one line (features p, p + 16, p + 32, ... of a group)
template <int G>
__device__ __forceinline__ void rq_high(float* y) {
    constexpr int V = G / 16;
    if constexpr (V > 1) rq_digit<V, V, 1, false>(y);
    if constexpr (V > 4) rq_digit<V, V, 4, false>(y);
}

template <int DT>
__device__ __forceinline__ void rq_load16(const char* row, int f0, int K, bool vec, float (&v)[16]) {
    constexpr int ES = DtInfo<DT>::ES;
    if (vec && f0 + 16 <= K) {
#pragma unroll
        for (int i = 0; i < 16 * ES / 16; ++i) ld16<DT>(row + (size_t) f0 * ES + 16 * i, v + i * (16 / ES));
    } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = f0 + e < K ? ld1<DT>(row, (size_t) (f0 + e)) : 0.0f;
    }
}

// x [M, K] (row stride K elements) -> xq int8 [M, Kp] (row stride Kp = K rounded up to 16, zeros past K), rs [M].
// vec: 16-byte loads allowed (K * element size a multiple of 16, x 16-byte aligned). G = 0: no rotation.
template <int DT, int G>
__global__ void __launch_bounds__(kRqThreads) rotq_rows(const void* __restrict__ x, int M, int K, int Kp, int vec,
                                                        int8_t* __restrict__ xq, float* __restrict__ rs) {
    constexpr int ES = DtInfo<DT>::ES;
    extern __shared__ float4 rq_smem4[];
    float* sv = reinterpret_cast<float*>(rq_smem4);
    __shared__ float wmax[2][kRqThreads / 32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int nwin = (K + kRqWin - 1) / kRqWin;
    const bool resident = K <= kRqResident;
    int parity = 0;
    for (int r = blockIdx.x; r < M; r += gridDim.x, parity ^= 1) {
        const char* xr = static_cast<const char*>(x) + (size_t) r * K * ES;
        // window w of the row, rotated, into shared memory; returns this thread's max |value| over what it finished
        auto rotate = [&](int w) -> float {
            float* base = sv + (resident ? w * kRqWinPad : 0);
            float v[16];
            rq_load16<DT>(xr, w * kRqWin + 16 * t, K, vec != 0, v);
            float m = 0.0f;
            if constexpr (G > 0) rq_low<G>(v);
            if constexpr (G > 0 && G <= 16) {
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = __fmul_rn(v[e], RqDigits<G>::NORM);
            }
            if constexpr (G <= 16) {
#pragma unroll
                for (int e = 0; e < 16; ++e) m = fmaxf(m, fabsf(v[e]));
            }
            float4* s4 = reinterpret_cast<float4*>(base + rq_pad(16 * t));
#pragma unroll
            for (int i = 0; i < 4; ++i) s4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            if constexpr (G >= 32) {
                constexpr int V = G / 16, LINES = kRqWin / V;
                __syncthreads();
#pragma unroll 1
                for (int L = t; L < LINES; L += kRqThreads) {
                    const int f = (L / 16) * G + (L % 16);
                    float y[V];
#pragma unroll
                    for (int j = 0; j < V; ++j) y[j] = base[rq_pad(f + 16 * j)];
                    rq_high<G>(y);
#pragma unroll
                    for (int j = 0; j < V; ++j) {
                        y[j] = __fmul_rn(y[j], RqDigits<G>::NORM);
                        m = fmaxf(m, fabsf(y[j]));
                        base[rq_pad(f + 16 * j)] = y[j];
                    }
                }
                __syncthreads();
            }
            return m;
        };
        float m = 0.0f;
        for (int w = 0; w < nwin; ++w) m = fmaxf(m, rotate(w));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) wmax[parity][warp] = m;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kRqThreads / 32; ++i) m = fmaxf(m, wmax[parity][i]);
        const float scale = fmaxf(__fdiv_rn(m, 127.0f), 1e-30f);
        if (t == 0) rs[r] = scale;
        for (int w = 0; w < nwin; ++w) {
            if (!resident) rotate(w);   // every thread, so that the barriers inside match
            const int f0 = w * kRqWin + 16 * t;
            if (f0 >= Kp) continue;
            const float4* s4 = reinterpret_cast<const float4*>(sv + (resident ? w * kRqWinPad : 0) + rq_pad(16 * t));
            uint32_t packed[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 q4 = s4[i];
                const float vv[4] = {q4.x, q4.y, q4.z, q4.w};
                uint32_t word = 0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float qf = fminf(127.0f, fmaxf(-128.0f, rintf(__fdiv_rn(vv[k], scale))));
                    word |= ((uint32_t) (__float2int_rn(qf) & 0xff)) << (8 * k);
                }
                packed[i] = word;
            }
            *reinterpret_cast<uint4*>(xq + (size_t) r * Kp + f0) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
    }
}

template <int DT, int G>
inline cudaError_t launch_rotq_g(const void* x, int M, int K, int Kp, bool vec, int8_t* xq, float* rs, int n_sm,
                                 cudaStream_t st) {
    const int nwin = (K + kRqWin - 1) / kRqWin;
    const int smem = (K <= kRqResident ? nwin : 1) * kRqWinPad * (int) sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(rotq_rows<DT, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const int grid = std::min(M, n_sm * 8);
    rotq_rows<DT, G><<<grid, kRqThreads, smem, st>>>(x, M, K, Kp, vec ? 1 : 0, xq, rs);
    return cudaGetLastError();
}

template <int DT>
inline cudaError_t launch_rotq(const void* x, int M, int K, int Kp, int group, int8_t* xq, float* rs, int n_sm,
                               cudaStream_t st) {
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ((size_t) K * DtInfo<DT>::ES) % 16 == 0;
    switch (group) {
        case 0: return launch_rotq_g<DT, 0>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        case 2: return launch_rotq_g<DT, 2>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        case 4: return launch_rotq_g<DT, 4>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        case 8: return launch_rotq_g<DT, 8>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        case 16: return launch_rotq_g<DT, 16>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        case 32: return launch_rotq_g<DT, 32>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        case 64: return launch_rotq_g<DT, 64>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        case 128: return launch_rotq_g<DT, 128>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        case 256: return launch_rotq_g<DT, 256>(x, M, K, Kp, vec, xq, rs, n_sm, st);
        default: return cudaErrorInvalidValue;
    }
}

// w [N, K] -> [N, Kp] with zeros past K, for a K that is not a multiple of 16 (TMA wants 16-byte row strides)
__global__ void pad_rows_i8(const int8_t* __restrict__ w, int N, int K, int Kp, int8_t* __restrict__ dst) {
    const size_t total = (size_t) N * Kp;
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t) gridDim.x * blockDim.x) {
        const size_t n = i / Kp, k = i % Kp;
        dst[i] = k < (size_t) K ? w[n * K + k] : 0;
    }
}

// ---- the int8 GEMM ----------------------------------------------------------------------------------------------------
constexpr int kLinBM = 128, kLinBN = 256, kLinBK = 128;   // tile rows, tile columns, bytes (= int8 values) per K slice
constexpr int kLinStages = 4;
constexpr int kLinThreads = 192;                          // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kLinTileA = kLinBM * kLinBK, kLinTileB = kLinBN * kLinBK, kLinStage = kLinTileA + kLinTileB;
constexpr int kLinOffBar = kLinStages * kLinStage;
constexpr int kLinSmem = kLinOffBar + 256 + 1024;         // + barriers, TMEM slot, abort flag; + 1 KB for the alignment
constexpr int kLinTmemCols = 2 * kLinBN;                  // two accumulators
constexpr int kErrLinear = 32;
constexpr uint32_t kLinIdesc = idesc(kFmtS32, kFmtS8, kFmtS8, 0, 0, kLinBM, kLinBN);

struct LinArgs {
    int M, N, nkb;               // rows, outputs, 128-byte K slices
    int n_mb, n_nb, band;        // 128-row blocks, 256-column blocks, column blocks per raster band
    const float* rs;             // row scales [M]
    const float* ws;             // weight scales: [N] when per_n, else [1]
    int per_n;
    const float* bias;           // [N] or NULL
    void* out;                   // [M, N], row stride N, in out_dt
    int out_dt, out_vec;         // out_vec: 16-byte stores allowed (N and the base checked on the host)
    int* err;                    // device error word
    unsigned long long wait_ns;  // limit of every wait
};

// Tile order: bands of `band` column blocks (a slice of W that stays in L2), row blocks one after the other inside a
// band and the band's column blocks fastest, so the CTAs running at once share a few row blocks of x_q and the band.
__device__ __forceinline__ void lin_tile(const LinArgs& a, int tile, int& mb, int& nb) {
    const int per_band = a.n_mb * a.band;
    const int bi = tile / per_band, local = tile - bi * per_band;
    const int nb0 = bi * a.band;
    const int bw = min(a.band, a.n_nb - nb0);
    mb = local / bw;
    nb = nb0 + local % bw;
}

__device__ __forceinline__ void lin_store32(const LinArgs& a, int row, int n0, const float (&y)[32]) {
    const int cnt = min(32, a.N - n0);
    const size_t off = (size_t) row * a.N + n0;
    if (a.out_dt == F32) {
        float* o = static_cast<float*>(a.out) + off;
        if (a.out_vec && cnt == 32) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                reinterpret_cast<float4*>(o)[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < cnt) o[j] = y[j];
        }
        return;
    }
    const bool h = a.out_dt == F16;
    uint16_t* o = static_cast<uint16_t*>(a.out) + off;
    if (a.out_vec && cnt == 32) {
        uint32_t p[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            if (h) {
                const __half2 v = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
                p[i] = *reinterpret_cast<const uint32_t*>(&v);
            } else {
                const __nv_bfloat162 v = __floats2bfloat162_rn(y[2 * i], y[2 * i + 1]);
                p[i] = *reinterpret_cast<const uint32_t*>(&v);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(o)[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < cnt) o[j] = h ? __half_as_ushort(__float2half_rn(y[j])) : __bfloat16_as_ushort(__float2bfloat16_rn(y[j]));
    }
}

// one tile's accumulator (this warp's 32 rows, 256 columns) -> out
__device__ __forceinline__ void lin_epilogue(const LinArgs& a, uint32_t taddr, int row, int n_base) {
    const bool row_ok = row < a.M;
    float rsf = 0.0f;
    if (row_ok) rsf = a.per_n ? a.rs[row] : __fmul_rn(a.rs[row], a.ws[0]);
#pragma unroll 1
    for (int cc = 0; cc < kLinBN / 32; ++cc) {
        const int n0 = n_base + cc * 32;
        if (n0 >= a.N) break;    // the same for the whole warp
        uint32_t r[32];
        tmem_ld32(taddr + cc * 32, r);
        tmem_wait_ld();
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int n = n0 + j;
            float v = __fmul_rn(__int2float_rn((int) r[j]), rsf);
            if (a.per_n) v = __fmul_rn(v, n < a.N ? __ldg(a.ws + n) : 0.0f);
            if (a.bias) v = __fadd_rn(v, n < a.N ? __ldg(a.bias + n) : 0.0f);
            y[j] = v;
        }
        if (row_ok) lin_store32(a, row, n0, y);
    }
}

// tmA: x_q, dims (Kp, M), box (128, 128); tmB: W, dims (Kp, N), box (128, 256); both 128-byte swizzled, zeros outside
__global__ void __launch_bounds__(kLinThreads, 1) i8gemm(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmB, const LinArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kLinOffBar);   // [stage]: both tiles of a K slice landed
    uint64_t* empty = full + kLinStages;                              // [stage]: the MMAs reading it are complete
    uint64_t* acc_full = empty + kLinStages;                          // [accumulator]: a tile's MMAs are complete
    uint64_t* acc_empty = acc_full + 2;                               // [accumulator], one arrival per epilogue warp
    uint64_t* done = acc_empty + 2;                                   // every MMA of the CTA is complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = a.n_mb * a.n_nb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kLinStages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(acc_full + b, 1); mbar_init(acc_empty + b, 4); }
        mbar_init(done, 1);
        *abort = *reinterpret_cast<volatile int*>(a.err) != 0;   // a failed launch before: no work in this CTA
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kLinTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto fail = [&]() {
        atomicOr(a.err, kErrLinear);
        *abort = 1;
    };
    const bool skip = *abort != 0;

    if (skip) {
    } else if (warp == 0) {
        // ---------------- TMA producer (one lane) ----------------
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            bool ok = true;
            int it = 0;   // K slices issued, over all tiles of this CTA
            for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
                if (*reinterpret_cast<volatile int*>(a.err) != 0) { *abort = 1; ok = false; break; }
                int mb, nb;
                lin_tile(a, tile, mb, nb);
                for (int kb = 0; kb < a.nkb; ++kb, ++it) {
                    const int s = it % kLinStages;
                    if (it >= kLinStages && !mbar_wait(empty + s, ((it / kLinStages) - 1) & 1, a.wait_ns, abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = sm + s * kLinStage;
                    mbar_expect_tx(full + s, kLinStage);
                    tma_load_2d(st, &tmA, full + s, kb * kLinBK, mb * kLinBM);
                    tma_load_2d(st + kLinTileA, &tmB, full + s, kb * kLinBK, nb * kLinBN);
                }
            }
            if (!ok) fail();
            // no copy may still be landing in shared memory when the CTA ends: the last slice issued into each stage
            for (int s = 0; s < kLinStages; ++s) {
                if (it - 1 < s) continue;
                const int last = s + kLinStages * ((it - 1 - s) / kLinStages);
                mbar_wait(full + s, (last / kLinStages) & 1, a.wait_ns, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (the whole warp runs the loop, one elected lane issues) ----------------
        bool ok = true;
        int it = 0, tc = 0;
        for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++tc) {
            const int buf = tc & 1;
            // the epilogue has read this accumulator's previous tile
            if (tc >= 2 && !warp_wait(acc_empty + buf, ((tc >> 1) - 1) & 1, a.wait_ns, abort)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d = tmem + buf * kLinBN;
            for (int kb = 0; kb < a.nkb; ++kb, ++it) {
                const int s = it % kLinStages;
                if (!warp_wait(full + s, (it / kLinStages) & 1, a.wait_ns, abort, 64)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sa = smem_u32(sm + s * kLinStage), sb = sa + kLinTileA;
#pragma unroll
                for (int kk = 0; kk < kLinBK / 32; ++kk)
                    mma_ss_w<true>(d, sdesc(sa + kk * 32, 16, 1024), sdesc(sb + kk * 32, 16, 1024), kLinIdesc,
                                   (kb | kk) != 0);
                mma_commit_w(empty + s);
            }
            if (!ok) break;
            mma_commit_w(acc_full + buf);
        }
        if (!ok && lane == 0) fail();
        // nothing may still be writing tensor memory or reading shared memory when the CTA ends
        mma_commit_w(done);
        warp_wait(done, 0, a.wait_ns, nullptr);
    } else {
        // ---------------- epilogue: warps 2-5, TMEM lanes 32 * (warp % 4) .. + 31 ----------------
        const int q = warp & 3;
        bool ok = true;
        int tc = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tc) {
            const int buf = tc & 1;
            if (!warp_wait(acc_full + buf, (tc >> 1) & 1, a.wait_ns, abort)) { ok = false; break; }
            tc_fence_after();
            int mb, nb;
            lin_tile(a, tile, mb, nb);
            lin_epilogue(a, tmem + buf * kLinBN + ((uint32_t) (32 * q) << 16), mb * kLinBM + 32 * q + lane, nb * kLinBN);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + buf);
        }
        if (!ok && lane == 0) fail();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kLinTmemCols);
    }
}

// A 2-D int8 map: dims (cols, rows), row stride in bytes, box (128, box_rows), 128-byte swizzle, zeros outside.
inline std::string make_i8_map(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int64_t row_bytes,
                               int box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return "cuTensorMapEncodeTiled is not available from the driver";
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15)) return "not 16-byte aligned";
    const cuuint64_t dims[2] = {(cuuint64_t) cols, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t) kLinBK, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return "cuTensorMapEncodeTiled failed (" + std::to_string((int) r) + ")";
    return {};
}

inline cudaError_t launch_i8gemm(const CUtensorMap& ta, const CUtensorMap& tb, const LinArgs& a, int n_sm, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(i8gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, kLinSmem);
    if (e != cudaSuccess) return e;
    const int tiles = a.n_mb * a.n_nb;
    i8gemm<<<std::min(tiles, n_sm), kLinThreads, kLinSmem, st>>>(ta, tb, a);
    return cudaGetLastError();
}

}  // namespace h3
