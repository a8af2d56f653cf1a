// prepass.cuh - the Sage pre-pass for sm_100a (kernels/h3sycl.cpp:1704-1764 of the reference), bit-exact with it:
//
//   kmean     kmean[h*D+d] = (((0 + k_0) + k_1) + ... + k_{S-1}) / (float) S: one fp32 chain per channel in token order
//             (the reference's loop, kernels/h3sycl.cpp:1733-1737). A chain cannot be split without changing its bits,
//             so the work is shaped around it: a TMA ring streams 256-token x 64-channel tiles of k into shared memory
//             (160 KB in flight per CTA) while 64 threads run the 64 chains over each tile, adding the 16-bit values
//             with the mixed-precision add (no separate conversion).
//   quant     per (head, 64-row block): m = max|x - mean|, inv = m > 0 ? 127/m : 0, scale = m/127,
//             q = clamp(round(x * inv), -127, 127), round half away from zero (kernels/h3sycl.cpp:1738-1761).
//             One CTA per block; the 64 x D values are read once with 16-byte loads and held in registers (as the raw
//             chunks) between the absmax and the quantisation.
//   to_half   any dt -> half [H, S, D] (kernels/h3sycl.cpp:1762-1764), only where the attention cannot read in place;
//             rows padded to Dp >= D features (16-byte rows for the TMA maps; the padding is never read: the maps cover
//             the first D features and TMA fills the rest of a box with zeros).
//
// All arithmetic uses the round-to-nearest intrinsics (__fadd_rn, __fsub_rn, __fmul_rn, __fdiv_rn), which the compiler
// never fuses into FMAs, so the results do not depend on contraction.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "attn_common.cuh"
#include "ptx.cuh"

namespace h3 {

template <int DT> struct DtInfo;
template <> struct DtInfo<F32> { static constexpr int ES = 4; };
template <> struct DtInfo<F16> { static constexpr int ES = 2; };
template <> struct DtInfo<BF16> { static constexpr int ES = 2; };

template <int DT>
__device__ __forceinline__ float ld1(const void* p, size_t i) {
    if constexpr (DT == F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    else if constexpr (DT == BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    else return reinterpret_cast<const float*>(p)[i];
}
// 16 bytes (as loaded) -> 16/ES floats
template <int DT>
__device__ __forceinline__ void cvt16(const uint4 u, float* out) {
    if constexpr (DT == F32) {
        out[0] = __uint_as_float(u.x); out[1] = __uint_as_float(u.y); out[2] = __uint_as_float(u.z); out[3] = __uint_as_float(u.w);
    } else {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint16_t lo = (uint16_t) (w[i] & 0xffffu), hi = (uint16_t) (w[i] >> 16);
            if constexpr (DT == F16) {
                out[2 * i] = __half2float(__ushort_as_half(lo));
                out[2 * i + 1] = __half2float(__ushort_as_half(hi));
            } else {
                out[2 * i] = __uint_as_float((uint32_t) lo << 16);
                out[2 * i + 1] = __uint_as_float((uint32_t) hi << 16);
            }
        }
    }
}
// 16 bytes at p -> 16/ES floats
template <int DT>
__device__ __forceinline__ void ld16(const void* p, float* out) {
    cvt16<DT>(*reinterpret_cast<const uint4*>(p), out);
}

// ---- K mean, TMA ring ----------------------------------------------------------------------------------------------
constexpr int kMeanCh = 64;          // channels per CTA: 128-byte rows of 16-bit k per token, two chain warps
// The TMA ring of one K-mean CTA: 5 tiles of 32 KB. Beside the q quantiser, whose traffic lengthens the loads' latency,
// a chain drained 3 tiles before the next arrived: measured at configs[3], the K mean beside the q quantiser took
// 214.8 us with 96 KB, 196 us with 160 or 192 KB (167 us alone with any), the pre-pass 331 against 310.5 us.
constexpr int kMeanRingBytes = 160 * 1024;
constexpr int kMeanThreads = 32 + kMeanCh;   // warp 0: producer; warps 1-2: one thread per chain

template <int DT>
struct MeanCfg {
    static constexpr int ROWS = DtInfo<DT>::ES == 2 ? 256 : 128;   // tokens per tile: 32 KB
    static constexpr int TILE = kMeanCh * ROWS * DtInfo<DT>::ES;
    static constexpr int NS = kMeanRingBytes / TILE;
    static constexpr int SMEM = NS * TILE + 2 * NS * 8 + 16 + 128;
};

// One k element as stored (16-bit types: the raw bits) and the chain's add of it: for f16 / bf16 the sm_100
// mixed-precision add (f32 + f16 / bf16 in one instruction, one rounding). Widening a 16-bit value to fp32 is exact,
// so the result has the bits of __fadd_rn(sum, (float) x); the separate conversion it replaces runs at a quarter of
// the fp32 rate and set the chain's pace (measured at S = 47,232: 199-201 us per K mean with it, 164-166 without).
template <int DT> struct KElem { using T = float; };
template <> struct KElem<F16> { using T = unsigned short; };
template <> struct KElem<BF16> { using T = unsigned short; };
template <int DT>
__device__ __forceinline__ typename KElem<DT>::T ld_k(const uint8_t* tile, int i) {
    return reinterpret_cast<const typename KElem<DT>::T*>(tile)[i];
}
template <int DT>
__device__ __forceinline__ float add_k(float s, typename KElem<DT>::T x) {
    float d;
    if constexpr (DT == F16) asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(x), "f"(s));
    else if constexpr (DT == BF16) asm("add.rn.f32.bf16 %0, %1, %2;" : "=f"(d) : "h"(x), "f"(s));
    else d = __fadd_rn(s, x);
    return d;
}

// map: 2-D over k, dims (H*D channels, S tokens), row stride in bytes, box (kMeanCh, MeanCfg<DT>::ROWS), no swizzle.
// The chain of each thread adds its channel's values of a tile in token order; the next 16 values are read from
// shared memory while the current 16 are added (the chain's dependent adds set the pace).
template <int DT>
__global__ void __launch_bounds__(kMeanThreads) kmean_tma(const __grid_constant__ CUtensorMap map, int S, int C,
                                                          float* kmean, int* err, unsigned long long wait_ns) {
    using M = MeanCfg<DT>;
    constexpr int ROWS = M::ROWS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + M::NS * M::TILE);
    uint64_t* empty = full + M::NS;
    volatile int* abort = reinterpret_cast<volatile int*>(empty + M::NS);
    const int c0 = blockIdx.x * kMeanCh;
    const int ntile = (S + ROWS - 1) / ROWS;
    if (threadIdx.x == 0) {
        // a stage is free once both chain warps have added it
        for (int i = 0; i < M::NS; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, 2); }
        *abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        if (threadIdx.x == 0) {
            tma_prefetch_desc(&map);
            int last[M::NS];
            for (int i = 0; i < M::NS; ++i) last[i] = -1;
            bool ok = true;
            for (int t = 0; t < ntile; ++t) {
                const int st = t % M::NS;
                if (t >= M::NS && !mbar_wait(empty + st, ((t / M::NS) - 1) & 1, wait_ns, abort)) { ok = false; break; }
                mbar_expect_tx(full + st, M::TILE);
                tma_load_2d(sm + st * M::TILE, &map, full + st, c0, t * ROWS);
                last[st] = t;
            }
            if (!ok) { atomicOr(err, kErrPrepass); *abort = 1; }
            for (int i = 0; i < M::NS; ++i)
                if (last[i] >= 0) mbar_wait(full + i, (last[i] / M::NS) & 1, wait_ns, nullptr);
        }
        __syncwarp();
    } else {
        const int c = threadIdx.x - 32;
        float sum = 0.0f;
        bool ok = true;
        for (int t = 0; t < ntile; ++t) {
            const int st = t % M::NS;
            // the whole warp agrees, so that it leaves the loop together (the __syncwarp below needs every lane)
            if (!warp_wait(full + st, (t / M::NS) & 1, wait_ns, abort)) { ok = false; break; }
            const uint8_t* tile = sm + st * M::TILE;
            const int rows = min(ROWS, S - t * ROWS);
            if (rows == ROWS) {
                typename KElem<DT>::T a[16], b[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) a[i] = ld_k<DT>(tile, i * kMeanCh + c);
#pragma unroll
                for (int r = 0; r < ROWS; r += 32) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) b[i] = ld_k<DT>(tile, (r + 16 + i) * kMeanCh + c);
#pragma unroll
                    for (int i = 0; i < 16; ++i) sum = add_k<DT>(sum, a[i]);
                    if (r + 32 < ROWS) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) a[i] = ld_k<DT>(tile, (r + 32 + i) * kMeanCh + c);
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) sum = add_k<DT>(sum, b[i]);
                }
            } else {
                for (int r = 0; r < rows; ++r) sum = add_k<DT>(sum, ld_k<DT>(tile, r * kMeanCh + c));
            }
            __syncwarp();
            if ((c & 31) == 0) mbar_arrive(empty + st);
        }
        if (!ok) { atomicOr(err, kErrPrepass); *abort = 1; }
        else if (c0 + c < C) kmean[c0 + c] = __fdiv_rn(sum, (float) S);
    }
    __syncthreads();
}

// The TMA map kmean_tma reads k through (k 16-byte aligned, the row stride a multiple of 16 bytes); false when the
// driver cannot make it (the caller then uses kmean_plain).
template <int DT>
inline bool make_kmean_map(CUtensorMap* map, const void* k, int C, int64_t S, int64_t stride) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t) C, (cuuint64_t) S};
    const cuuint64_t strides[1] = {(cuuint64_t) (stride * DtInfo<DT>::ES)};
    const cuuint32_t box[2] = {(cuuint32_t) kMeanCh, (cuuint32_t) MeanCfg<DT>::ROWS};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType ty = DT == F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                 : DT == BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    return enc(map, ty, 2, const_cast<void*>(k), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Any alignment: one thread per channel reading k directly (the fallback for strides TMA cannot take).
template <int DT>
__global__ void kmean_plain(const void* k, int S, int C, long long stride, float* kmean) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float sum = 0.0f;
    for (int t = 0; t < S; ++t) sum = __fadd_rn(sum, ld1<DT>(k, (size_t) t * (size_t) stride + (size_t) c));
    kmean[c] = __fdiv_rn(sum, (float) S);
}

// The K mean of C channels over S tokens of k (row stride `stride` elements) on stream st: kmean_tma, or kmean_plain
// where TMA cannot read k.
template <int DT>
inline cudaError_t launch_kmean(const void* k, int64_t S, int C, int64_t stride, float* kmean, int* err,
                                unsigned long long wait_ns, cudaStream_t st) {
    const bool tma_ok = (reinterpret_cast<uintptr_t>(k) & 15) == 0 && (stride * DtInfo<DT>::ES) % 16 == 0;
    CUtensorMap map;
    if (tma_ok && make_kmean_map<DT>(&map, k, C, S, stride)) {
        using M = MeanCfg<DT>;
        const cudaError_t e = cudaFuncSetAttribute(kmean_tma<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, M::SMEM);
        if (e != cudaSuccess) return e;
        kmean_tma<DT><<<(C + kMeanCh - 1) / kMeanCh, kMeanThreads, M::SMEM, st>>>(map, (int) S, C, kmean, err, wait_ns);
    } else {
        kmean_plain<DT><<<(C + 127) / 128, 128, 0, st>>>(k, (int) S, C, (long long) stride, kmean);
    }
    return cudaGetLastError();
}

// ---- quantiser -----------------------------------------------------------------------------------------------------
// The packed pair type of a 16-bit element type, its NaN and its exact widening.
template <int DT> struct Half2Of;
template <> struct Half2Of<F16> {
    using T = __half2;
    static __device__ __forceinline__ T nan2() { return __halves2half2(__ushort_as_half(0x7E00), __ushort_as_half(0x7E00)); }
    static __device__ __forceinline__ float2 to_float2(T v) { return __half22float2(v); }
};
template <> struct Half2Of<BF16> {
    using T = __nv_bfloat162;
    static __device__ __forceinline__ T nan2() {
        return __halves2bfloat162(__ushort_as_bfloat16(0x7FC0), __ushort_as_bfloat16(0x7FC0));
    }
    static __device__ __forceinline__ float2 to_float2(T v) { return __bfloat1622float2(v); }
};
constexpr int kQuantThreads = 128;

// grid (nb, H); src rows at element stride `stride`, head h at column h*D; dst int8 [H, S, D]; scales [H, nb].
// VEC: 16-byte loads (every row start 16-byte aligned, checked on the host).
template <int DT, int D, bool VEC>
__global__ void __launch_bounds__(kQuantThreads) quant_rows(const void* src, int S, long long stride, const float* mean,
                                                            int8_t* dst, float* scales, int nb) {
    constexpr int EPC = 16 / DtInfo<DT>::ES;          // elements per 16-byte chunk
    constexpr int CPR = D / EPC;                      // chunks per row
    constexpr int NCH = 64 * CPR / kQuantThreads;     // chunks per thread
    static_assert(kQuantThreads % CPR == 0, "a thread keeps one column chunk");
    const int b = blockIdx.x, h = blockIdx.y;
    const int r0 = b * 64, rows = min(64, S - r0);
    const int col = (threadIdx.x % CPR) * EPC;        // this thread's first feature
    const int rsub = threadIdx.x / CPR;               // first row; then every kQuantThreads/CPR rows
    constexpr int RSTEP = kQuantThreads / CPR;
    float mu[EPC];
#pragma unroll
    for (int e = 0; e < EPC; ++e) mu[e] = mean ? mean[h * D + col + e] : 0.0f;
    // the raw 16-byte chunks stay in registers between the two passes (half the registers of the converted floats,
    // so more CTAs, and more loads in flight, per SM); each pass converts them the same way
    uint4 raw[NCH];
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int r = rsub + i * RSTEP;
        raw[i] = make_uint4(0, 0, 0, 0);
        if (r < rows) {
            const size_t base = (size_t) (r0 + r) * (size_t) stride + (size_t) (h * D + col);
            if constexpr (VEC) {
                raw[i] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(src) + base * DtInfo<DT>::ES);
            } else {
                uint8_t* rb = reinterpret_cast<uint8_t*>(&raw[i]);
#pragma unroll
                for (int e = 0; e < 16; ++e) rb[e] = reinterpret_cast<const uint8_t*>(src)[base * DtInfo<DT>::ES + e];
            }
        }
    }
    float m = 0.0f;
    if constexpr (DtInfo<DT>::ES == 2) {
        // x -> __fsub_rn(x, mean) is monotone, so over this thread's rows the largest |x - mean| of a channel is at the
        // channel's largest or smallest value: those two, found on the 16-bit values (exact, two channels per
        // instruction), are all that is converted and subtracted. The min/max start at NaN and skip NaN, as fmaxf
        // below skips a NaN |x - mean|, so the result has the bits of the per-element loop.
        using T2 = typename Half2Of<DT>::T;
        T2 hi[EPC / 2], lo[EPC / 2];
#pragma unroll
        for (int p = 0; p < EPC / 2; ++p) hi[p] = lo[p] = Half2Of<DT>::nan2();
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
            if (rsub + i * RSTEP < rows) {
                const T2* v = reinterpret_cast<const T2*>(&raw[i]);
#pragma unroll
                for (int p = 0; p < EPC / 2; ++p) {
                    hi[p] = __hmax2(hi[p], v[p]);
                    lo[p] = __hmin2(lo[p], v[p]);
                }
            }
        }
#pragma unroll
        for (int p = 0; p < EPC / 2; ++p) {
            const float2 a = Half2Of<DT>::to_float2(hi[p]), c = Half2Of<DT>::to_float2(lo[p]);
            m = fmaxf(m, fabsf(__fsub_rn(a.x, mu[2 * p])));
            m = fmaxf(m, fabsf(__fsub_rn(c.x, mu[2 * p])));
            m = fmaxf(m, fabsf(__fsub_rn(a.y, mu[2 * p + 1])));
            m = fmaxf(m, fabsf(__fsub_rn(c.y, mu[2 * p + 1])));
        }
    } else {
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
            if (rsub + i * RSTEP < rows) {
                float x[EPC];
                ld16<DT>(&raw[i], x);
#pragma unroll
                for (int e = 0; e < EPC; ++e) m = fmaxf(m, fabsf(__fsub_rn(x[e], mu[e])));
            }
        }
    }
    // block absmax
    __shared__ float red[kQuantThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int w = 1; w < kQuantThreads / 32; ++w) m = fmaxf(m, red[w]);
    const float inv = m > 0.0f ? __fdiv_rn(127.0f, m) : 0.0f;
    if (threadIdx.x == 0) scales[(size_t) h * nb + b] = __fdiv_rn(m, 127.0f);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int r = rsub + i * RSTEP;
        if (r < rows) {
            float x[EPC];
            ld16<DT>(&raw[i], x);
            int8_t qv[EPC];
#pragma unroll
            for (int e = 0; e < EPC; ++e)
                qv[e] = (int8_t) fminf(127.0f, fmaxf(-127.0f, roundf(__fmul_rn(__fsub_rn(x[e], mu[e]), inv))));
            int8_t* d = dst + ((size_t) h * S + r0 + r) * D + col;
            if constexpr (EPC == 8) *reinterpret_cast<uint2*>(d) = *reinterpret_cast<const uint2*>(qv);
            else *reinterpret_cast<uint32_t*>(d) = *reinterpret_cast<const uint32_t*>(qv);
        }
    }
}

// any dt, token rows -> half [H, S, D] (one sequence)
template <int DT>
__global__ void to_half_hsd(const void* src, int S, int H, int D, long long stride, __half* dst, int Dp) {
    const size_t n = (size_t) S * H * D;
    for (size_t i = blockIdx.x * (size_t) blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) {
        const size_t d = i % D, t = (i / D) % S, hh = i / ((size_t) D * S);
        dst[(hh * S + t) * Dp + d] = __float2half_rn(ld1<DT>(src, t * (size_t) stride + hh * D + d));
    }
}

}  // namespace h3
