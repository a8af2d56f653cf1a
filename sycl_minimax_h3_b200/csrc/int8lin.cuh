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

// clamp(rint(v / scale), -128, 127) with the quotient rounded to float first (v / scale, then rint), as the reference
// computes it, without a division per value: y = v * inv (inv = 1/scale correctly rounded) is within 1.5 units in the
// last place of the rounded quotient q (|y - q| <= 1.5 * 2^-23 * |q| < 2.3e-5 for |q| <= 128), so rint(y) = rint(q)
// unless y lies within 2^-14 of a half-integer; those few values take the exact quotient. Clamping before rounding
// is the same as after (the bounds are integers). Rounding to an integer, half to even: adding 1.5 * 2^23 leaves the
// integer in the low mantissa bits.
__device__ __forceinline__ int rq_code(float v, float inv, float scale) {
    const float y = fminf(127.0f, fmaxf(-128.0f, __fmul_rn(v, inv)));
    const float t = __fadd_rn(y, 12582912.0f);
    const float d = fabsf(__fsub_rn(y, __fsub_rn(t, 12582912.0f)));
    if (d > 0.5f - 6.103515625e-05f) {
        const float q = fminf(127.0f, fmaxf(-128.0f, rintf(__fdiv_rn(v, scale))));
        return __float2int_rn(q);
    }
    return __float_as_int(t) - 0x4B400000;
}

// 16 values -> their 16 int8 codes, 4 per word (rq_code's decision, checked once per chunk): with |v * inv| <= 127
// (the row scale bounds every value), the integer nearest the exact product v * inv sits in the low byte of
// t = 1.5 * 2^23 + v * inv (one rounding), whose bit pattern is 0x4B400000 plus the integer. That integer is rint of the
// rounded quotient v / scale unless the product lies within 2^-14 of a half (the quotient and the product differ by
// less than 1.2e-5 there); one predicate collects those values (and any NaN or infinity, whose difference is NaN), and
// such a chunk takes rq_code for every value.
__device__ __forceinline__ uint4 rq_codes16(const float (&v)[16], float inv, float scale) {
    uint32_t w[4];
    bool near = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t tb[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            // t = 1.5*2^23 + v*inv rounded once: the integer nearest v*inv (half to even) in the low bits; d = v*inv
            // minus that integer, rounded once
            const float t = __fmaf_rn(v[4 * i + k], inv, 12582912.0f);
            const float d = __fmaf_rn(v[4 * i + k], inv, -__fsub_rn(t, 12582912.0f));
            near |= !(fabsf(d) <= 0.5f - 6.103515625e-05f);
            tb[k] = __float_as_uint(t);
        }
        w[i] = __byte_perm(__byte_perm(tb[0], tb[1], 0x0040), __byte_perm(tb[2], tb[3], 0x0040), 0x5410);
    }
    if (near) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t tb[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) tb[k] = (uint32_t) rq_code(v[4 * i + k], inv, scale);
            w[i] = __byte_perm(__byte_perm(tb[0], tb[1], 0x0040), __byte_perm(tb[2], tb[3], 0x0040), 0x5410);
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Offset (in floats) of feature f + 16 j from feature f in the padded shared-memory row, for f = g0 + p (p < 16) in a
// group of G >= 32 features starting at g0 (a multiple of G; G divides 256, so the group stays inside one block of 256)
__host__ __device__ constexpr int rq_line_off(int j) { return 16 * j + 4 * (j >> 1); }

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
                for (int e = 0; e < 16; e += 2) m = fmax3(m, fabsf(v[e]), fabsf(v[e + 1]));
            }
            float4* s4 = reinterpret_cast<float4*>(base + rq_pad(16 * t));
#pragma unroll
            for (int i = 0; i < 4; ++i) s4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            if constexpr (G >= 32) {
                constexpr int V = G / 16, LINES = kRqWin / V;
                __syncthreads();
#pragma unroll 1
                for (int L = t; L < LINES; L += kRqThreads) {
                    float* lp = base + rq_pad((L / 16) * G + (L % 16));
                    float y[V];
#pragma unroll
                    for (int j = 0; j < V; ++j) y[j] = lp[rq_line_off(j)];
                    rq_high<G>(y);
#pragma unroll
                    for (int j = 0; j < V; ++j) {
                        y[j] = __fmul_rn(y[j], RqDigits<G>::NORM);
                        lp[rq_line_off(j)] = y[j];
                    }
#pragma unroll
                    for (int j = 0; j < V; j += 2) m = fmax3(m, fabsf(y[j]), fabsf(y[j + 1]));
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
        const float inv = __frcp_rn(scale);
        if (t == 0) rs[r] = scale;
        for (int w = 0; w < nwin; ++w) {
            if (!resident) rotate(w);   // every thread, so that the barriers inside match
            const int f0 = w * kRqWin + 16 * t;
            if (f0 >= Kp) continue;
            const float4* s4 = reinterpret_cast<const float4*>(sv + (resident ? w * kRqWinPad : 0) + rq_pad(16 * t));
            float vv[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 q4 = s4[i];
                vv[4 * i] = q4.x; vv[4 * i + 1] = q4.y; vv[4 * i + 2] = q4.z; vv[4 * i + 3] = q4.w;
            }
            *reinterpret_cast<uint4*>(xq + (size_t) r * Kp + f0) = rq_codes16(vv, inv, scale);
        }
    }
}

// The common case: 16-byte loads allowed and the row (K <= NW * 4096 features) kept in shared memory. The next row's
// 16-byte pieces are loaded into registers while the current row is rotated (NW windows of one 16-feature chunk per
// thread), so each CTA has two rows in flight and the load latency stays hidden. Two CTA barriers per row: after the
// chunks are stored (before the high digits read other threads' chunks) and after the row's maxima; none for groups
// of 16 and less, where each thread only reads back its own chunks.
template <int DT, int G, int NW>
__global__ void __launch_bounds__(kRqThreads) rotq_fast(const void* __restrict__ x, int M, int K, int Kp,
                                                        int8_t* __restrict__ xq, float* __restrict__ rs) {
    constexpr int ES = DtInfo<DT>::ES;
    constexpr int PC = ES, FPP = 16 / ES;   // 16-byte pieces per chunk, features per piece
    extern __shared__ float4 rq_smem4[];
    float* sv = reinterpret_cast<float*>(rq_smem4);
    __shared__ float wmax[2][kRqThreads / 32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int nwin = (K + kRqWin - 1) / kRqWin;
    uint4 nxt[NW][PC];
    auto fetch = [&](int r) {
        const char* xr = static_cast<const char*>(x) + (size_t) r * K * ES;
#pragma unroll
        for (int w = 0; w < NW; ++w)
#pragma unroll
            for (int i = 0; i < PC; ++i) {
                const int f = w * kRqWin + 16 * t + i * FPP;
                nxt[w][i] = (w < nwin && f + FPP <= K) ? __ldcs(reinterpret_cast<const uint4*>(xr + (size_t) f * ES))
                                                       : make_uint4(0, 0, 0, 0);
            }
    };
    int parity = 0;
    if (blockIdx.x < M) fetch(blockIdx.x);
    for (int r = blockIdx.x; r < M; r += gridDim.x, parity ^= 1) {
        uint4 cur[NW][PC];
#pragma unroll
        for (int w = 0; w < NW; ++w)
#pragma unroll
            for (int i = 0; i < PC; ++i) cur[w][i] = nxt[w][i];
        if (r + (int) gridDim.x < M) fetch(r + gridDim.x);
        float m = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            if (w >= nwin) break;
            float v[16];
#pragma unroll
            for (int i = 0; i < PC; ++i) cvt16<DT>(cur[w][i], v + i * FPP);
            if constexpr (G > 0) rq_low<G>(v);
            if constexpr (G > 0 && G <= 16) {
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = __fmul_rn(v[e], RqDigits<G>::NORM);
            }
            if constexpr (G <= 16) {
#pragma unroll
                for (int e = 0; e < 16; e += 2) m = fmax3(m, fabsf(v[e]), fabsf(v[e + 1]));
            }
            float4* s4 = reinterpret_cast<float4*>(sv + w * kRqWinPad + rq_pad(16 * t));
#pragma unroll
            for (int i = 0; i < 4; ++i) s4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
        if constexpr (G >= 32) {
            constexpr int V = G / 16, LINES = kRqWin / V;
            __syncthreads();
#pragma unroll 1
            for (int w = 0; w < nwin; ++w) {
                float* base = sv + w * kRqWinPad;
#pragma unroll 1
                for (int L = t; L < LINES; L += kRqThreads) {
                    float* lp = base + rq_pad((L / 16) * G + (L % 16));
                    float y[V];
#pragma unroll
                    for (int j = 0; j < V; ++j) y[j] = lp[rq_line_off(j)];
                    rq_high<G>(y);
#pragma unroll
                    for (int j = 0; j < V; ++j) {
                        y[j] = __fmul_rn(y[j], RqDigits<G>::NORM);
                        lp[rq_line_off(j)] = y[j];
                    }
#pragma unroll
                    for (int j = 0; j < V; j += 2) m = fmax3(m, fabsf(y[j]), fabsf(y[j + 1]));
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) wmax[parity][warp] = m;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kRqThreads / 32; ++i) m = fmaxf(m, wmax[parity][i]);
        const float scale = fmaxf(__fdiv_rn(m, 127.0f), 1e-30f);
        const float inv = __frcp_rn(scale);
        if (t == 0) rs[r] = scale;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const int f0 = w * kRqWin + 16 * t;
            if (w >= nwin || f0 >= Kp) break;
            const float4* s4 = reinterpret_cast<const float4*>(sv + w * kRqWinPad + rq_pad(16 * t));
            float vv[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 q4 = s4[i];
                vv[4 * i] = q4.x; vv[4 * i + 1] = q4.y; vv[4 * i + 2] = q4.z; vv[4 * i + 3] = q4.w;
            }
            *reinterpret_cast<uint4*>(xq + (size_t) r * Kp + f0) = rq_codes16(vv, inv, scale);
        }
    }
}

// persistent grid: as many CTAs as fit on the SMs at once (each then takes rows m, m + grid, ...)
template <typename Kern>
inline int rq_grid(Kern k, int smem, int M, int n_sm) {
    int per_sm = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kRqThreads, smem) != cudaSuccess || per_sm < 1) per_sm = 1;
    return std::min(M, n_sm * per_sm);
}

template <int DT, int G>
inline cudaError_t launch_rotq_g(const void* x, int M, int K, int Kp, bool vec, int8_t* xq, float* rs, int n_sm,
                                 cudaStream_t st) {
    const int nwin = (K + kRqWin - 1) / kRqWin;
    cudaError_t e;
    if (vec && nwin == 1) {
        const int smem = kRqWinPad * (int) sizeof(float);
        if ((e = cudaFuncSetAttribute(rotq_fast<DT, G, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
            return e;
        rotq_fast<DT, G, 1><<<rq_grid(rotq_fast<DT, G, 1>, smem, M, n_sm), kRqThreads, smem, st>>>(x, M, K, Kp, xq, rs);
        return cudaGetLastError();
    }
    if constexpr (DT != F32) {
        if (vec && nwin <= 4) {
            const int smem = nwin * kRqWinPad * (int) sizeof(float);
            if ((e = cudaFuncSetAttribute(rotq_fast<DT, G, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
                return e;
            rotq_fast<DT, G, 4><<<rq_grid(rotq_fast<DT, G, 4>, smem, M, n_sm), kRqThreads, smem, st>>>(x, M, K, Kp, xq, rs);
            return cudaGetLastError();
        }
    }
    // everything else (unaligned or odd rows, rows longer than 16384 features, float32 rows over 4096): rotq_rows
    const int smem = (K <= kRqResident ? nwin : 1) * kRqWinPad * (int) sizeof(float);
    if ((e = cudaFuncSetAttribute(rotq_rows<DT, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
        return e;
    rotq_rows<DT, G><<<rq_grid(rotq_rows<DT, G>, smem, M, n_sm), kRqThreads, smem, st>>>(x, M, K, Kp, vec ? 1 : 0, xq, rs);
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
constexpr int kLinOffCols = kLinOffBar + 256;             // staged scales and bias: [2 tiles][2][256] floats
constexpr int kLinSmem = kLinOffCols + 4 * kLinBN * 4 + 1024;   // + 1 KB for the alignment
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

// The tile's per-output scales and bias, staged in shared memory by the 128 epilogue threads (two columns each) before
// the accumulator is ready: the rescale then reads them as broadcast vector loads instead of one global load per value
// (which the compiler cannot move above the previous chunk's stores, so each chunk waited a full memory round trip).
constexpr int kLinEpiBar = 1;   // named barrier of the four epilogue warps
__device__ __forceinline__ void lin_stage(const LinArgs& a, float* sws, float* sb, int n_base, int et) {
#pragma unroll
    for (int i = et; i < kLinBN; i += 128) {
        const int n = n_base + i;
        sws[i] = (a.per_n && n < a.N) ? __ldg(a.ws + n) : 0.0f;
        sb[i] = (a.bias && n < a.N) ? __ldg(a.bias + n) : 0.0f;
    }
}

// one tile's accumulator (this warp's 32 rows, 256 columns) -> out; rsf = the row's scale (times the single weight
// scale), sws / sb = the staged per-output scales and bias
__device__ __forceinline__ void lin_epilogue(const LinArgs& a, uint32_t taddr, int row, int n_base, float rsf,
                                             const float* sws, const float* sb) {
    const bool row_ok = row < a.M;
#pragma unroll 1
    for (int cc = 0; cc < kLinBN / 32; ++cc) {
        const int n0 = n_base + cc * 32;
        if (n0 >= a.N) break;    // the same for the whole warp
        uint32_t r[32];
        tmem_ld32(taddr + cc * 32, r);
        tmem_wait_ld();
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) y[j] = __fmul_rn(__int2float_rn((int) r[j]), rsf);
        if (a.per_n) {
            const float4* w4 = reinterpret_cast<const float4*>(sws + cc * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 w = w4[i];
                y[4 * i] = __fmul_rn(y[4 * i], w.x);
                y[4 * i + 1] = __fmul_rn(y[4 * i + 1], w.y);
                y[4 * i + 2] = __fmul_rn(y[4 * i + 2], w.z);
                y[4 * i + 3] = __fmul_rn(y[4 * i + 3], w.w);
            }
        }
        if (a.bias) {
            const float4* b4 = reinterpret_cast<const float4*>(sb + cc * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 b = b4[i];
                y[4 * i] = __fadd_rn(y[4 * i], b.x);
                y[4 * i + 1] = __fadd_rn(y[4 * i + 1], b.y);
                y[4 * i + 2] = __fadd_rn(y[4 * i + 2], b.z);
                y[4 * i + 3] = __fadd_rn(y[4 * i + 3], b.w);
            }
        }
        if (row_ok) lin_store32(a, row, n0, y);
    }
}

// The epilogue role of both GEMM kernels (warps 2-5; et = 0..127): per tile, stage the columns' scales and bias, wait
// for the accumulator, write the rows, release the accumulator (one arrival per warp on `release`, a shared::cluster
// address). The four warps meet at a named barrier once per tile on every path: after a failure a warp goes on through
// its tiles without waiting or working, so the others never wait there for it.
__device__ __forceinline__ bool lin_epilogue_role(const LinArgs& a, int tile0, int stride, int rows_per_tile,
                                                  int row_off, uint32_t tmem, uint64_t* acc_full,
                                                  const uint32_t (&release)[2], float* stage, volatile int* abort) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, q = warp & 3, et = threadIdx.x - 64;
    const int tiles = a.n_mb * a.n_nb;
    const bool cols = a.per_n || a.bias;
    bool ok = true;
    int tc = 0;
    for (int tile = tile0; tile < tiles; tile += stride, ++tc) {
        const int buf = tc & 1;
        int mb, nb;
        lin_tile(a, tile, mb, nb);
        float* sws = stage + buf * 2 * kLinBN;
        float* sb = sws + kLinBN;
        const int row = mb * rows_per_tile + row_off + 32 * q + lane;
        float rsf = 0.0f;
        if (ok) {
            if (cols) lin_stage(a, sws, sb, nb * kLinBN, et);
            if (row < a.M) rsf = a.per_n ? a.rs[row] : __fmul_rn(a.rs[row], a.ws[0]);
            ok = warp_wait(acc_full + buf, (tc >> 1) & 1, a.wait_ns, abort);
        }
        if (cols) bar_sync(kLinEpiBar, 128);
        if (ok) {
            tc_fence_after();
            lin_epilogue(a, tmem + buf * kLinBN + ((uint32_t) (32 * q) << 16), row, nb * kLinBN, rsf, sws, sb);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(buf ? release[1] : release[0]);
        }
    }
    return ok;
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
        const uint32_t rel[2] = {smem_u32(acc_empty), smem_u32(acc_empty + 1)};
        if (!lin_epilogue_role(a, blockIdx.x, gridDim.x, kLinBM, 0, tmem, acc_full, rel,
                               reinterpret_cast<float*>(sm + kLinOffCols), abort) && lane == 0)
            fail();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kLinTmemCols);
    }
}

// ---- the int8 GEMM on SM pairs (cta_group::2) ----------------------------------------------------------------------------
// A cluster of two CTAs computes 256 x 256 tiles: each CTA loads its own 128 rows of x_q and its half (128 rows) of the
// tile's 256 rows of W, 32 KB per K slice instead of 48 (the pair reads W's rows once between them), so 6 stages fit
// and the L2 traffic per MMA falls by a third. Rank 0 issues tcgen05.mma.cta_group::2 (M = 256) for both; each CTA's
// tensor memory holds its own 128 rows of the two accumulators, and its epilogue warps write those rows.
// Barriers: the stage's `full` and the accumulators' `acc_empty` live in rank 0 (both CTAs' copies and both epilogues
// count there); `empty`, `acc_full` and `done` in each CTA, signalled by rank 0's commits (one to each CTA).
constexpr int kL2Stages = 6;
constexpr int kL2TileA = 128 * kLinBK, kL2TileB = 128 * kLinBK, kL2Stage = kL2TileA + kL2TileB;
constexpr int kL2OffBar = kL2Stages * kL2Stage;
constexpr int kL2OffCols = kL2OffBar + 256;
constexpr int kL2Smem = kL2OffCols + 4 * kLinBN * 4 + 1024;
constexpr uint32_t kL2Idesc = idesc(kFmtS32, kFmtS8, kFmtS8, 0, 0, 256, kLinBN);

// tmA: x_q, dims (Kp, M), box (128, 128); tmB: W, dims (Kp, N), box (128, 128); a.n_mb counts 256-row blocks
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kLinThreads, 1)
    i8gemm2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const LinArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kL2OffBar);     // [stage] (rank 0's count): both CTAs' copies
    uint64_t* empty = full + kL2Stages;                                // [stage]: the MMAs reading it are complete
    uint64_t* acc_full = empty + kL2Stages;                            // [accumulator]: a tile's MMAs are complete
    uint64_t* acc_empty = acc_full + 2;                                // [accumulator] (rank 0's count): 8 warps
    uint64_t* done = acc_empty + 2;                                    // every MMA of the pair is complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint32_t* issued = tmem_slot + 2;                                  // K slices this CTA's producer issued
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool lead = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int tiles = a.n_mb * a.n_nb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kL2Stages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(acc_full + b, 1); mbar_init(acc_empty + b, 8); }
        mbar_init(done, 1);
        *abort = *reinterpret_cast<volatile int*>(a.err) != 0;   // a failed launch before: no work in this CTA
        *issued = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kLinTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();   // both CTAs' barriers are initialised before either CTA touches the other's
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto fail = [&]() {
        atomicOr(a.err, kErrLinear);
        *abort = 1;
    };
    const bool skip = *abort != 0;

    if (skip) {
    } else if (warp == 0) {
        // ---------------- TMA producer, both CTAs (one lane each) ----------------
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            bool ok = true;
            int it = 0;
            for (int tile = pair; ok && tile < tiles; tile += npairs) {
                if (*reinterpret_cast<volatile int*>(a.err) != 0) { *abort = 1; ok = false; break; }
                int mb, nb;
                lin_tile(a, tile, mb, nb);
                for (int kb = 0; kb < a.nkb; ++kb, ++it) {
                    const int s = it % kL2Stages;
                    if (it >= kL2Stages && !mbar_wait(empty + s, ((it / kL2Stages) - 1) & 1, a.wait_ns, abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = sm + s * kL2Stage;
                    const uint32_t bar0 = mapa_shared(smem_u32(full + s), 0);
                    if (lead) mbar_expect_tx(full + s, 2 * kL2Stage);
                    tma_load_2d_pair(st, &tmA, bar0, kb * kLinBK, mb * 256 + (int) rank * 128);
                    tma_load_2d_pair(st + kL2TileA, &tmB, bar0, kb * kLinBK, nb * kLinBN + (int) rank * 128);
                }
            }
            if (!ok) fail();
            *issued = (uint32_t) it;
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer: rank 0's warp 1 for the pair ----------------
        if (lead) {
            bool ok = true;
            int it = 0, tc = 0;
            for (int tile = pair; ok && tile < tiles; tile += npairs, ++tc) {
                const int buf = tc & 1;
                if (tc >= 2 && !warp_wait(acc_empty + buf, ((tc >> 1) - 1) & 1, a.wait_ns, abort)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + buf * kLinBN;
                for (int kb = 0; kb < a.nkb; ++kb, ++it) {
                    const int s = it % kL2Stages;
                    if (!warp_wait(full + s, (it / kL2Stages) & 1, a.wait_ns, abort, 64)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(sm + s * kL2Stage), sb = sa + kL2TileA;
#pragma unroll
                    for (int kk = 0; kk < kLinBK / 32; ++kk)
                        mma_pair_i8_w(d, sdesc(sa + kk * 32, 16, 1024), sdesc(sb + kk * 32, 16, 1024), kL2Idesc, (kb | kk) != 0);
                    mma_commit_pair_w(mapa_shared(smem_u32(empty + s), 0));
                    mma_commit_pair_w(mapa_shared(smem_u32(empty + s), 1));
                }
                if (!ok) break;
                mma_commit_pair_w(mapa_shared(smem_u32(acc_full + buf), 0));
                mma_commit_pair_w(mapa_shared(smem_u32(acc_full + buf), 1));
            }
            if (!ok && lane == 0) fail();
            mma_commit_pair_w(mapa_shared(smem_u32(done), 0));
            warp_wait(done, 0, a.wait_ns, nullptr);
        }
    } else {
        // ---------------- epilogue: warps 2-5 of both CTAs, each CTA its 128 rows of the tile ----------------
        const uint32_t rel[2] = {mapa_shared(smem_u32(acc_empty), 0), mapa_shared(smem_u32(acc_empty + 1), 0)};
        if (!lin_epilogue_role(a, pair, npairs, 256, (int) rank * 128, tmem, acc_full, rel,
                               reinterpret_cast<float*>(sm + kL2OffCols), abort) && lane == 0)
            fail();
    }

    // Neither CTA leaves while the other may still reach its memory. Every copy of both CTAs counts on rank 0's `full`
    // barriers: rank 0 waits there for the last slice either producer issued into each stage (the producers may have
    // stopped at different slices after a failure), then both pass the second cluster barrier.
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (lead && threadIdx.x == 0) {
        const int n = (int) max(*issued, ld_shared_cluster(mapa_shared(smem_u32(issued), 1)));
        for (int s = 0; s < kL2Stages; ++s) {
            if (n - 1 < s) continue;
            const int last = s + kL2Stages * ((n - 1 - s) / kL2Stages);
            mbar_wait(full + s, (last / kL2Stages) & 1, a.wait_ns, nullptr);
        }
    }
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kLinTmemCols);
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

// The GEMM behind h3s_int8_linear: i8gemm2 on SM pairs; H3S_LIN_KERNEL=1 selects i8gemm (one SM per 128 x 256 tile),
// kept for comparison. The weight map's box is 128 rows for i8gemm2, 256 for i8gemm (lin_weight_rows).
inline bool lin_pairs() {
    static const bool pairs = [] {
        const char* e = std::getenv("H3S_LIN_KERNEL");
        return !(e && std::atoi(e) == 1);
    }();
    return pairs;
}
inline int lin_weight_rows() { return lin_pairs() ? 128 : kLinBN; }
inline int lin_rows_per_tile() { return lin_pairs() ? 256 : kLinBM; }

inline cudaError_t launch_i8gemm(const CUtensorMap& ta, const CUtensorMap& tb, const LinArgs& a, int n_sm, cudaStream_t st) {
    const int tiles = a.n_mb * a.n_nb;
    if (lin_pairs()) {
        cudaError_t e = cudaFuncSetAttribute(i8gemm2, cudaFuncAttributeMaxDynamicSharedMemorySize, kL2Smem);
        if (e != cudaSuccess) return e;
        i8gemm2<<<2 * std::min(tiles, n_sm / 2), kLinThreads, kL2Smem, st>>>(ta, tb, a);
    } else {
        cudaError_t e = cudaFuncSetAttribute(i8gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, kLinSmem);
        if (e != cudaSuccess) return e;
        i8gemm<<<std::min(tiles, n_sm), kLinThreads, kLinSmem, st>>>(ta, tb, a);
    }
    return cudaGetLastError();
}

}  // namespace h3
