// rmsrope.cuh - per-head RMS norm + rotary position rotation, in place: the step that runs on q and k right before the
// attention in every denoiser block (engine/h3-core/src/dit.rs:347-348; kernels/h3sycl.cpp:1276-1376 of the reference).
//
// Per (token m, head h), over the head's D features x_i (row m at element m*stride, head h at h*D):
//   s   = ((0 + x_0*x_0) + x_1*x_1) + ... + x_{D-1}*x_{D-1}        (fp32, feature order, every step rounded)
//   inv = rsqrt(s / D + eps)                                       (correctly rounded, __frsqrt_rn)
//   pairs (i, rot/2 + i), i < rot/2:  a = (x_i*inv)*w_i, b = (x_{rot/2+i}*inv)*w_{rot/2+i},
//                                     x_i <- a*cos - b*sin, x_{rot/2+i} <- b*cos + a*sin   with (cos, sin) = cs[m, i]
//   features from rot on:             x_i <- (x_i*inv)*w_i
// each result rounded to the element type (RNE). Every product and sum uses the _rn intrinsics, which the compiler
// never fuses into FMAs, so the bits do not depend on contraction (the CPU restatement in the oracle matches them).
//
// HBM-bound: one read and one write of each row. A CTA takes 32 consecutive (token, head) rows: it stages them in
// shared memory with coalesced 16-byte loads (a head's D features are contiguous; consecutive heads of a token are
// adjacent), each thread then works on its own row there, and the CTA writes the rows back the same way. Rows are
// padded by 16 bytes in shared memory, so a warp's 16-byte accesses to 32 rows spread over the banks. Layouts the
// staging cannot take (unaligned rows, D not a multiple of a 16-byte chunk, D > 256) go through rms_rope_plain, one
// thread per row reading global memory directly, with the same arithmetic.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "prepass.cuh"

namespace h3 {

// (token, head) rows per CTA, one per thread. Small CTAs, many per SM, so that their load, work and store phases
// overlap: measured at configs[3] (one fp16 tensor, 0.77 GB read and written) 172 us with 32 rows, 176 with 64 and
// 183 with 128 (4.50, 4.39 and 4.23 TB/s); 16 loads in flight per thread instead of 8: 201 us (fewer CTAs fit).
constexpr int kRopeRows = 32;
constexpr int kRopeMaxD = 256;

template <int DT>
__device__ __forceinline__ float rr_ld(const uint8_t* p) {
    if constexpr (DT == F16) return __half2float(*reinterpret_cast<const __half*>(p));
    else if constexpr (DT == BF16) return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
    else return *reinterpret_cast<const float*>(p);
}
template <int DT>
__device__ __forceinline__ void rr_st(uint8_t* p, float v) {
    if constexpr (DT == F16) *reinterpret_cast<__half*>(p) = __float2half_rn(v);
    else if constexpr (DT == BF16) *reinterpret_cast<__nv_bfloat16*>(p) = __float2bfloat16_rn(v);
    else *reinterpret_cast<float*>(p) = v;
}

// The arithmetic on one row whose element i sits at row + i*ES (global or shared memory).
template <int DT>
__device__ __forceinline__ void rr_row(uint8_t* row, int m, int D, int half, int rot, const float* __restrict__ w,
                                       float eps, const float* __restrict__ cs) {
    constexpr int ES = DtInfo<DT>::ES;
    float s = 0.0f;
    for (int i = 0; i < D; ++i) {
        const float v = rr_ld<DT>(row + i * ES);
        s = __fadd_rn(s, __fmul_rn(v, v));
    }
    const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(s, (float) D), eps));
    const float* c = cs + (size_t) m * half * 2;
    for (int j = 0; j < half; ++j) {
        const float a = __fmul_rn(__fmul_rn(rr_ld<DT>(row + j * ES), inv), __ldg(w + j));
        const float b = __fmul_rn(__fmul_rn(rr_ld<DT>(row + (half + j) * ES), inv), __ldg(w + half + j));
        const float co = __ldg(c + 2 * j), si = __ldg(c + 2 * j + 1);
        rr_st<DT>(row + j * ES, __fsub_rn(__fmul_rn(a, co), __fmul_rn(b, si)));
        rr_st<DT>(row + (half + j) * ES, __fadd_rn(__fmul_rn(b, co), __fmul_rn(a, si)));
    }
    for (int i = rot; i < D; ++i)
        rr_st<DT>(row + i * ES, __fmul_rn(__fmul_rn(rr_ld<DT>(row + i * ES), inv), __ldg(w + i)));
}

// 16 bytes of shared memory <-> EPC floats (RNE narrowing, two values per instruction)
template <int DT>
__device__ __forceinline__ void rr_ld16(const uint8_t* p, float* v) { ld16<DT>(p, v); }
template <int DT>
__device__ __forceinline__ void rr_st16(uint8_t* p, const float* v) {
    if constexpr (DT == F32) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if constexpr (DT == F16) {
                const __half2 h = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
                w[e] = *reinterpret_cast<const uint32_t*>(&h);
            } else {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
                w[e] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}
// Pairs of scalar round-to-nearest products and sums. (The packed f32x2 forms, __fmul2_rn / __fadd2_rn or PTX
// mul.rn.f32x2 / add.rn.f32x2, were measured on the B200 to give different bits from the scalar forms in this
// multiply-then-add arithmetic for about 1.5 % of the rotated values, so the bit-exact path stays scalar.)
__device__ __forceinline__ float2 rr_mul2(float2 a, float2 b) { return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y)); }
__device__ __forceinline__ float2 rr_add2(float2 a, float2 b) { return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)); }

// n floats (a multiple of 4) from a 16-byte aligned global address
template <int N>
__device__ __forceinline__ void ldg_f4(const float* __restrict__ p, float (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p) + i);
        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
}

// rr_row on a row in shared memory, 16 bytes at a time: a warp's 16-byte accesses to 32 padded rows take the minimum
// number of bank wavefronts (2-byte accesses would conflict 4 ways); the weight and the (cos, sin) table come in
// 16-byte loads; the arithmetic is rr_row's, operation for operation. Needs rot/2 and rot multiples of 16/ES and
// 16-byte aligned w and cs.
template <int DT>
__device__ __forceinline__ void rr_row_chunks(uint8_t* row, int m, int D, int half, int rot, const float* __restrict__ w,
                                              float eps, const float* __restrict__ cs) {
    constexpr int ES = DtInfo<DT>::ES;
    constexpr int EPC = 16 / ES;
    float s = 0.0f;
    for (int i = 0; i < D; i += EPC) {
        float v[EPC];
        rr_ld16<DT>(row + i * ES, v);
#pragma unroll
        for (int e = 0; e < EPC; e += 2) {
            const float2 q = rr_mul2(make_float2(v[e], v[e + 1]), make_float2(v[e], v[e + 1]));
            s = __fadd_rn(s, q.x);
            s = __fadd_rn(s, q.y);
        }
    }
    const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(s, (float) D), eps));
    const float2 inv2 = make_float2(inv, inv);
    const float* c = cs + (size_t) m * half * 2;
    for (int j = 0; j < half; j += EPC) {
        float va[EPC], vb[EPC], wa[EPC], wb[EPC], cc[2 * EPC];
        rr_ld16<DT>(row + j * ES, va);
        rr_ld16<DT>(row + (half + j) * ES, vb);
        ldg_f4<EPC>(w + j, wa);
        ldg_f4<EPC>(w + half + j, wb);
        ldg_f4<2 * EPC>(c + 2 * j, cc);
#pragma unroll
        for (int e = 0; e < EPC; e += 2) {
            const float2 a = rr_mul2(rr_mul2(make_float2(va[e], va[e + 1]), inv2), make_float2(wa[e], wa[e + 1]));
            const float2 b = rr_mul2(rr_mul2(make_float2(vb[e], vb[e + 1]), inv2), make_float2(wb[e], wb[e + 1]));
            const float2 co = make_float2(cc[2 * e], cc[2 * e + 2]), si = make_float2(cc[2 * e + 1], cc[2 * e + 3]);
            const float2 nsi = make_float2(-si.x, -si.y);
            // a*cos - b*sin = a*cos + b*(-sin), exactly (negation is exact, rounding is symmetric)
            const float2 na = rr_add2(rr_mul2(a, co), rr_mul2(b, nsi));
            const float2 nb = rr_add2(rr_mul2(b, co), rr_mul2(a, si));
            va[e] = na.x; va[e + 1] = na.y;
            vb[e] = nb.x; vb[e + 1] = nb.y;
        }
        rr_st16<DT>(row + j * ES, va);
        rr_st16<DT>(row + (half + j) * ES, vb);
    }
    for (int i = rot; i < D; i += EPC) {
        float v[EPC], wv[EPC];
        rr_ld16<DT>(row + i * ES, v);
        ldg_f4<EPC>(w + i, wv);
#pragma unroll
        for (int e = 0; e < EPC; e += 2) {
            const float2 y = rr_mul2(rr_mul2(make_float2(v[e], v[e + 1]), inv2), make_float2(wv[e], wv[e + 1]));
            v[e] = y.x; v[e + 1] = y.y;
        }
        rr_st16<DT>(row + i * ES, v);
    }
}

// Staged through shared memory: rows 16-byte aligned, D * ES a multiple of 16, D <= kRopeMaxD.
template <int DT>
__global__ void __launch_bounds__(kRopeRows) rms_rope_staged(uint8_t* x, long long rows, int H, int D, long long stride,
                                                             const float* __restrict__ w, float eps,
                                                             const float* __restrict__ cs, int rot) {
    constexpr int ES = DtInfo<DT>::ES;
    extern __shared__ __align__(16) uint8_t tile[];
    const int rb = D * ES;                 // bytes of a row
    const int pitch = rb + 16;             // padded row in shared memory
    const int cpr = rb / 16;               // 16-byte chunks per row
    __shared__ long long row_off[kRopeRows];   // byte offset of each row: one 64-bit division per thread, not per chunk
    const long long r0 = (long long) blockIdx.x * kRopeRows;
    const int nrows = (int) min((long long) kRopeRows, rows - r0);
    int m = 0;
    if ((int) threadIdx.x < nrows) {
        const long long r = r0 + threadIdx.x;
        m = (int) (r / H);
        row_off[threadIdx.x] = ((long long) m * stride + (r - (long long) m * H) * D) * ES;
    }
    __syncthreads();
    // 8 loads in flight per thread before their shared-memory stores (one at a time, a thread would wait out the
    // memory latency per 16 bytes)
    const int nchunks = nrows * cpr;
    const bool pow2 = (cpr & (cpr - 1)) == 0;
    const int sh = __ffs(cpr) - 1;
    auto split = [&](int c, int& r, int& k) {
        r = pow2 ? c >> sh : c / cpr;
        k = c - r * cpr;
    };
    for (int c0 = threadIdx.x; c0 < nchunks; c0 += 8 * kRopeRows) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = c0 + u * kRopeRows;
            if (c < nchunks) {
                int r, k;
                split(c, r, k);
                v[u] = *reinterpret_cast<const uint4*>(x + row_off[r] + k * 16);
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = c0 + u * kRopeRows;
            if (c < nchunks) {
                int r, k;
                split(c, r, k);
                *reinterpret_cast<uint4*>(tile + r * pitch + k * 16) = v[u];
            }
        }
    }
    __syncthreads();
    if ((int) threadIdx.x < nrows) {
        constexpr int EPC = 16 / ES;
        if ((rot / 2) % EPC == 0 && rot % EPC == 0 && ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(cs)) & 15) == 0)
            rr_row_chunks<DT>(tile + threadIdx.x * pitch, m, D, rot / 2, rot, w, eps, cs);
        else
            rr_row<DT>(tile + threadIdx.x * pitch, m, D, rot / 2, rot, w, eps, cs);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < nchunks; c += kRopeRows) {
        int r, k;
        split(c, r, k);
        *reinterpret_cast<uint4*>(x + row_off[r] + k * 16) = *reinterpret_cast<const uint4*>(tile + r * pitch + k * 16);
    }
}

// Any layout: one thread per row, global memory directly.
template <int DT>
__global__ void rms_rope_plain(uint8_t* x, long long rows, int H, int D, long long stride, const float* __restrict__ w,
                               float eps, const float* __restrict__ cs, int rot) {
    constexpr int ES = DtInfo<DT>::ES;
    const long long r = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    rr_row<DT>(x + ((r / H) * stride + (r % H) * D) * ES, (int) (r / H), D, rot / 2, rot, w, eps, cs);
}

template <int DT>
cudaError_t launch_rms_rope(void* x, long long M, int H, int D, long long stride, const float* w, float eps,
                            const float* cs, int rot, cudaStream_t st) {
    constexpr int ES = DtInfo<DT>::ES;
    const long long rows = M * H;
    const bool staged = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (stride * ES) % 16 == 0 && (D * ES) % 16 == 0 &&
                        D <= kRopeMaxD;
    if (staged) {
        const int smem = kRopeRows * (D * ES + 16);
        cudaError_t e = cudaFuncSetAttribute(rms_rope_staged<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        // all of the SM's unified L1/shared storage as shared memory, so that many CTAs stay resident and their load,
        // work and store phases overlap; a carveout sized for one CTA left the SMs waiting on one CTA's memory latency
        // at a time
        e = cudaFuncSetAttribute(rms_rope_staged<DT>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        rms_rope_staged<DT><<<(unsigned) ((rows + kRopeRows - 1) / kRopeRows), kRopeRows, smem, st>>>(
            static_cast<uint8_t*>(x), rows, H, D, stride, w, eps, cs, rot);
    } else {
        rms_rope_plain<DT><<<(unsigned) ((rows + 127) / 128), 128, 0, st>>>(static_cast<uint8_t*>(x), rows, H, D, stride,
                                                                         w, eps, cs, rot);
    }
    return cudaGetLastError();
}

}  // namespace h3
