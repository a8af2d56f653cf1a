// causal.cuh - causal attention with grouped heads, for the text encoder's short sequences (engine/h3-core/src/te.rs
// :340-346; kernels/h3sycl.cpp:870-898 of the reference).
//
// Per query head h and query i, over the keys j <= i of key/value head g = h / (Hq/Hkv), all in fp32 between the loads
// and the store, as the reference does (it never rounds the weights):
//   s = (q_i . k_j) / sqrt(D);  mn = max(m, s);  a = exp(m - mn);  e = exp(s - mn);
//   acc = acc * a + e * v_j;    l = l * a + e;   m = mn;            out_i = acc / l   (rounded to the element type)
//
// One warp per (query, head): lane t holds features t, t+32, ... of q, acc and the rows it reads; a dot product is the
// lanes' partial sums combined by shuffles. The dot products of four keys are formed together (independent), then the
// four updates run in key order, each with the arithmetic above (expf, the accurate exponential). This runs on CUDA
// cores on purpose: the sequences are short (the prompt), the semantics keep every weight in fp32 (a tensor-core P.V
// would round them), and the encoder runs once per generation.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "prepass.cuh"

namespace h3 {

constexpr int kCausalWarps = 4;          // (query, head) pairs per CTA
constexpr int kCausalMaxPer = 8;         // features per lane: D <= 256

template <int DT, int PER>
__global__ void __launch_bounds__(32 * kCausalWarps) attn_causal(const void* __restrict__ q, const void* __restrict__ k,
                                                                 const void* __restrict__ v, int L, int Hq, int Hkv, int D,
                                                                 long long qs, long long kvs, void* __restrict__ out,
                                                                 float scale) {
    const int lane = threadIdx.x & 31;
    const long long pair = (long long) blockIdx.x * kCausalWarps + (threadIdx.x >> 5);
    if (pair >= (long long) L * Hq) return;
    // the longest queries first: later query rows sit in the lower block indices
    const int h = (int) (pair % Hq), i = L - 1 - (int) (pair / Hq);
    const int g = h / (Hq / Hkv);
    float qv[PER], acc[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const int d = lane + 32 * u;
        qv[u] = d < D ? ld1<DT>(q, (size_t) i * qs + (size_t) h * D + d) : 0.0f;
        acc[u] = 0.0f;
    }
    const size_t koff = (size_t) g * D;
    float m = -INFINITY, l = 0.0f;
    auto dot = [&](int j) {
        float p = 0.0f;
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int d = lane + 32 * u;
            if (d < D) p = fmaf(qv[u], ld1<DT>(k, (size_t) j * kvs + koff + d), p);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
        return p * scale;
    };
    auto update = [&](int j, float s) {
        const float mn = fmaxf(m, s);
        const float a = expf(m - mn), e = expf(s - mn);
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int d = lane + 32 * u;
            const float vd = d < D ? ld1<DT>(v, (size_t) j * kvs + koff + d) : 0.0f;
            acc[u] = acc[u] * a + e * vd;
        }
        l = l * a + e;
        m = mn;
    };
    int j = 0;
    for (; j + 4 <= i + 1; j += 4) {
        const float s0 = dot(j), s1 = dot(j + 1), s2 = dot(j + 2), s3 = dot(j + 3);
        update(j, s0);
        update(j + 1, s1);
        update(j + 2, s2);
        update(j + 3, s3);
    }
    for (; j <= i; ++j) update(j, dot(j));
    const float inv = 1.0f / l;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const int d = lane + 32 * u;
        if (d >= D) continue;
        const size_t o = (size_t) i * Hq * D + (size_t) h * D + d;
        const float y = acc[u] * inv;
        if constexpr (DT == F16) reinterpret_cast<__half*>(out)[o] = __float2half_rn(y);
        else if constexpr (DT == BF16) reinterpret_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(y);
        else reinterpret_cast<float*>(out)[o] = y;
    }
}

template <int DT>
cudaError_t launch_causal(const void* q, const void* k, const void* v, int L, int Hq, int Hkv, int D, long long qs,
                          long long kvs, void* out, cudaStream_t st) {
    const long long pairs = (long long) L * Hq;
    const unsigned grid = (unsigned) ((pairs + kCausalWarps - 1) / kCausalWarps);
    const float scale = 1.0f / sqrtf((float) D);
    const int per = (D + 31) / 32;
    if (per <= 2) attn_causal<DT, 2><<<grid, 32 * kCausalWarps, 0, st>>>(q, k, v, L, Hq, Hkv, D, qs, kvs, out, scale);
    else if (per <= 4) attn_causal<DT, 4><<<grid, 32 * kCausalWarps, 0, st>>>(q, k, v, L, Hq, Hkv, D, qs, kvs, out, scale);
    else attn_causal<DT, kCausalMaxPer><<<grid, 32 * kCausalWarps, 0, st>>>(q, k, v, L, Hq, Hkv, D, qs, kvs, out, scale);
    return cudaGetLastError();
}

}  // namespace h3
