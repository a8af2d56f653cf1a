// sage_ref.cpp - CPU restatement of the MiniMax-H3 denoiser self-attention path (maxfridbe/sycl_minimax_h3).
//
// TEST INFRASTRUCTURE ONLY. Nothing in the product (libh3cuda.so, libh3sage.so, the Python package) links, loads or
// calls this file. It is the checker used by tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline leg and
// `--impl reference` arm.
//
// What it restates, and from where (paths inside the reference project):
//   dtype helpers      kernels/h3sycl.cpp:42-63     bf16 <-> f32 on bits, f32 -> half (round to nearest even)
//   K channel mean     kernels/h3sycl.cpp:1733-1737 kmean[h*D+d] = (((0 + k_0) + k_1) + ... + k_{S-1}) / (float) S
//   Q / K quantiser    kernels/h3sycl.cpp:1738-1761 per (head, 64-row block): m = max|x - mean|, inv = m>0 ? 127/m : 0,
//                                                   scale = m/127, q = clamp(round(x*inv), -127, 127), round half away
//   V relayout         kernels/h3sycl.cpp:1762-1764 v -> half [H, S, D]
//   Sage core          kernels/sage.cpp:41-52       (ARK kernel, un-vendored): softmax(q.k * qs * ks * scale) v,
//                                                   int8 dots with int32 sums, fp32 softmax, P in half, fp32 P.V
//   output relayout    kernels/h3sycl.cpp:1769-1771 half [H, S, D] -> out_dt [S, H*D] (through half)
//   fp16 fused SDPA    kernels/h3sycl.cpp:1464-1500 MatMul -> f32 scores, x f32 scale, SoftMax -> f16 P,
//                                                   MatMul(P, v) -> f16   (oneDNN 3.12 graph, un-vendored)
//   dispatcher         kernels/h3sycl.cpp:1779-1798 Sage when S >= sage_min_s (8192) and D in {64, 128}, else SDPA
//   int8 ConvRot lin.  kernels/h3sycl.cpp:404-652   per row: Hadamard rotation per group, digit by digit in the order
//                                                   of the fused kernel (:404-470), scale = max(max|x_rot|/127, 1e-30),
//                                                   q = clamp(rint(x_rot/scale), -128, 127), int32 dots, then
//                                                   acc * (scale*ws) [or (acc*scale)*ws[n]] + bias (:573-599);
//                      engine/h3-core/src/reference.rs:37-82   the dense restatement as written (x_rot = x . H)
//   causal GQA attn    kernels/h3sycl.cpp:870-898   per (head, query i): online softmax over keys j <= i in fp32,
//                                                   s = (q.k) * 1/sqrt(D), exp, acc = acc*a + e*v, out = acc / l
//   RMS norm + RoPE    kernels/h3sycl.cpp:1276-1376 per (token, head): s = sum of v*v in feature order,
//                                                   inv = rsqrt(s/D + eps) (correctly rounded here), pairs
//                                                   (i, rot/2 + i) scaled (x*inv)*w then rotated by (cos, sin),
//                                                   the rest scaled; rounded back to the element type in place
//
// Parity status: the dtype helpers are pinned to the reference's own known-answer tests (engine/h3-core/src/dtype.rs
// :137-155). The quantiser and the attention arithmetic are UNPINNED: the reference has no test or fixture for them
// and cannot be built here (SYCL + oneDNN + un-vendored ARK/sycl-tla). "Bit-exact" for the quantiser therefore means
// bit-exact with this strict-IEEE restatement of the source order (build with -ffp-contract=off, no -ffast-math).
// The int8 linear is checked against the reference's own tests of it (engine/h3-core/src/reference.rs:101-127: the
// Hadamard matrix is orthonormal; the layer is within quantisation of a plain linear) and against the dense
// restatement of reference.rs below; the butterfly's rounding order is the reference's fused kernel's, read from the
// source (that kernel cannot run here).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include <atomic>
#include <thread>

namespace {

enum Dt : int { F32 = 0, F16 = 1, BF16 = 2 };
constexpr int kBlock = 64;   // quantisation block, kernels/h3sycl.cpp:1681 (kSageBlock)

inline float bits_f32(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t f32_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

// bf16 widening: the 16 bits are the top half of a float32 (kernels/h3sycl.cpp:43).
inline float bf16_to_f32(uint16_t b) { return bits_f32((uint32_t) b << 16); }
// bf16 narrowing: round to nearest even on the discarded 16 bits; inf/nan are truncated (kernels/h3sycl.cpp:44-49).
inline uint16_t f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7f800000u) == 0x7f800000u) return (uint16_t) (u >> 16);
    const uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t) ((u + 0x7fffu + lsb) >> 16);
}
// IEEE binary16 -> binary32, exact (normals, subnormals, zero, inf, nan).
inline float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0x1f) return bits_f32(sign | 0x7f800000u | (m << 13));
    if (e == 0) {
        if (m == 0) return bits_f32(sign);
        // subnormal: m * 2^-24, exact in float32
        const float v = (float) m * bits_f32(0x33800000u);   // 2^-24
        return sign ? -v : v;
    }
    return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}
// IEEE binary32 -> binary16, round to nearest even, overflow to inf (what (sycl::half) v does).
inline uint16_t f32_to_f16(float f) {
    const uint32_t u = f32_bits(f);
    const uint16_t sign = (uint16_t) ((u >> 16) & 0x8000u);
    const uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t) (sign | 0x7c00u | (a > 0x7f800000u ? 0x200u | ((a >> 13) & 0x3ffu) : 0));
    if (a >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u);            // rounds to >= 65520: inf
    if (a < 0x38800000u) {                                                 // below 2^-14: half subnormal or zero
        if (a < 0x33000000u) return sign;                                  // below 2^-25: rounds to zero
        const uint32_t e = a >> 23;                                        // 102 .. 112
        const uint32_t mant = (a & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;                                   // 14 .. 24
        uint32_t h = mant >> shift;
        const uint32_t rest = mant & ((1u << shift) - 1u), halfway = 1u << (shift - 1u);
        if (rest > halfway || (rest == halfway && (h & 1u))) ++h;
        return (uint16_t) (sign | h);
    }
    uint32_t h = ((a >> 23) - 112u) << 10 | ((a >> 13) & 0x3ffu);
    const uint32_t rest = a & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;             // a carry into the exponent is correct
    return (uint16_t) (sign | h);
}

inline float load(const void* p, int dt, size_t i) {
    switch (dt) {
        case F16: return f16_to_f32(((const uint16_t*) p)[i]);
        case BF16: return bf16_to_f32(((const uint16_t*) p)[i]);
        default: return ((const float*) p)[i];
    }
}
inline void store(void* p, int dt, size_t i, float v) {
    switch (dt) {
        case F16: ((uint16_t*) p)[i] = f32_to_f16(v); break;
        case BF16: ((uint16_t*) p)[i] = f32_to_bf16(v); break;
        default: ((float*) p)[i] = v;
    }
}
inline float half_round(float v) { return f16_to_f32(f32_to_f16(v)); }

// Work-sharing over [0, n): every host thread (H3_ORACLE_THREADS overrides) takes `chunk` items at a time.
int g_threads = 0;
int threads() {
    if (g_threads <= 0) {
        const char* e = std::getenv("H3_ORACLE_THREADS");
        g_threads = e ? std::atoi(e) : (int) std::thread::hardware_concurrency();
        if (g_threads <= 0) g_threads = 1;
    }
    return g_threads;
}
template <class F> void par_for(int64_t n, int64_t chunk, F&& f) {
    const int nt = (int) std::min<int64_t>(threads(), (n + chunk - 1) / chunk);
    if (nt <= 1) { for (int64_t i = 0; i < n; ++i) f(i, 0); return; }
    std::atomic<int64_t> next{0};
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; ++t)
        pool.emplace_back([&, t] {
            for (;;) {
                const int64_t b = next.fetch_add(chunk);
                if (b >= n) break;
                for (int64_t i = b; i < std::min(n, b + chunk); ++i) f(i, t);
            }
        });
    for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

// ---- dtype helpers, element-wise over n values ------------------------------------------------------------------
void orc_f32_to_f16(const float* x, uint16_t* y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = f32_to_f16(x[i]); }
void orc_f16_to_f32(const uint16_t* x, float* y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = f16_to_f32(x[i]); }
void orc_f32_to_bf16(const float* x, uint16_t* y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = f32_to_bf16(x[i]); }
void orc_bf16_to_f32(const uint16_t* x, float* y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = bf16_to_f32(x[i]); }

// How many host threads the oracle's loops use (H3_ORACLE_THREADS, else every hardware thread).
int orc_threads(void) { return threads(); }
void orc_set_threads(int n) { g_threads = n; }

// ---- K1: the channel mean of k over the sequence (kernels/h3sycl.cpp:1733-1737) -------------------------------
// One fp32 chain per channel, in token order, then one division by (float) S.
void orc_kmean(const void* k, int dt, int64_t S, int64_t H, int64_t D, int64_t stride, float* kmean) {
    par_for(H * D, 16, [&](int64_t c, int) {
        float sum = 0.0f;
        for (int64_t t = 0; t < S; ++t) sum += load(k, dt, (size_t) (t * stride + c));
        kmean[c] = sum / (float) S;
    });
}

// ---- K2/K3: int8 quantisation per (head, 64-row block) (kernels/h3sycl.cpp:1738-1761) --------------------------
// src rows of H*D values at element stride `stride`; mean [H*D] or NULL; dst int8 [H, S, D]; scales [H, nb].
void orc_quant(const void* src, int dt, int64_t S, int64_t H, int64_t D, int64_t stride, const float* mean,
               int8_t* dst, float* scales) {
    const int64_t nb = (S + kBlock - 1) / kBlock;
    par_for(H * nb, 8, [&](int64_t g, int) {
        const int64_t h = g / nb, b = g % nb, r0 = b * kBlock, rows = std::min<int64_t>(kBlock, S - r0);
        float m = 0.0f;
        for (int64_t r = r0; r < r0 + rows; ++r)
            for (int64_t d = 0; d < D; ++d) {
                const float x = load(src, dt, (size_t) (r * stride + h * D + d)) - (mean ? mean[h * D + d] : 0.0f);
                m = std::fmax(m, std::fabs(x));
            }
        const float inv = m > 0.0f ? 127.0f / m : 0.0f;
        scales[h * nb + b] = m / 127.0f;
        for (int64_t r = r0; r < r0 + rows; ++r)
            for (int64_t d = 0; d < D; ++d) {
                const float x = (load(src, dt, (size_t) (r * stride + h * D + d)) - (mean ? mean[h * D + d] : 0.0f)) * inv;
                dst[(h * S + r) * D + d] = (int8_t) std::min(127.0f, std::max(-127.0f, std::round(x)));
            }
    });
}

// ---- the whole Sage pre-pass (kernels/h3sycl.cpp:1704-1764) -------------------------------------------------------
// iq, ik int8 [H, S, D]; sc float [2*H*nb + H*D] = qs [H, nb], ks [H, nb], kmean [H*D] (kernels/h3sycl.cpp:1716-1718);
// hv half bits [H, S, D] (may be NULL).
void orc_sage_prepass(const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D,
                      int64_t stride, int8_t* iq, int8_t* ik, float* sc, uint16_t* hv) {
    const int64_t nb = (S + kBlock - 1) / kBlock;
    float* qs = sc;
    float* ks = sc + H * nb;
    float* kmean = sc + 2 * H * nb;
    orc_kmean(k, dt, S, H, D, stride, kmean);
    orc_quant(q, dt, S, H, D, stride, nullptr, iq, qs);
    orc_quant(k, dt, S, H, D, stride, kmean, ik, ks);
    if (hv)
        par_for(S, 64, [&](int64_t t, int) {
            for (int64_t h = 0; h < H; ++h)
                for (int64_t d = 0; d < D; ++d)
                    hv[(h * S + t) * D + d] = f32_to_f16(load(v, dt, (size_t) (t * stride + h * D + d)));
        });
}

// ---- Sage core (kernels/sage.cpp:41-52 semantics) on selected (head, row) pairs --------------------------------------
// iq, ik int8 [H, S, D]; hv half [H, S, D]; qs, ks [H, nb] for 64-row blocks; out half bits [n, D] for the n pairs
// (rows_h[i], rows_s[i]). score = (float) dot * (qs * ks * scale); fp32 softmax with the row max; p rounded to half;
// fp32 sum of p * v; divided by the fp32 sum of p; rounded to half. The rows are taken head by head, with that head's v
// widened to float once; the per-element order of every sum is the same as the plain loops'.
}  // extern "C"

namespace {
template <int DC>
inline int32_t dot_i8(const int8_t* __restrict a, const int8_t* __restrict b, int64_t D) {
    int32_t acc = 0;
    const int64_t n = DC > 0 ? DC : D;
    for (int64_t d = 0; d < n; ++d) acc += (int32_t) a[d] * (int32_t) b[d];
    return acc;
}
template <int DC>
inline void axpy(float* __restrict o, float p, const float* __restrict v, int64_t D) {
    const int64_t n = DC > 0 ? DC : D;
    for (int64_t d = 0; d < n; ++d) o[d] += p * v[d];
}
template <int DC>
void sage_rows_impl(const int8_t* iq, const int8_t* ik, const uint16_t* hv, const float* qs, const float* ks, int64_t S,
                    int64_t H, int64_t D, float scale, const int64_t* rows_h, const int64_t* rows_s, int64_t n,
                    uint16_t* out) {
    const int64_t nb = (S + kBlock - 1) / kBlock;
    std::vector<std::vector<int64_t>> by_head((size_t) H);
    for (int64_t i = 0; i < n; ++i) by_head[(size_t) rows_h[i]].push_back(i);
    const int nt = threads();
    std::vector<std::vector<float>> s_t((size_t) nt, std::vector<float>((size_t) S)), o_t((size_t) nt, std::vector<float>((size_t) D));
    std::vector<float> vf;
    for (int64_t h = 0; h < H; ++h) {
        const std::vector<int64_t>& rows = by_head[(size_t) h];
        if (rows.empty()) continue;
        vf.resize((size_t) (S * D));
        par_for(S, 256, [&](int64_t j, int) {
            for (int64_t d = 0; d < D; ++d) vf[(size_t) (j * D + d)] = f16_to_f32(hv[(h * S + j) * D + d]);
        });
        par_for((int64_t) rows.size(), 1, [&](int64_t ri, int t) {
            const int64_t i = rows[(size_t) ri], r = rows_s[i];
            std::vector<float>& s = s_t[(size_t) t];
            std::vector<float>& o = o_t[(size_t) t];
            const int8_t* qr = iq + (h * S + r) * D;
            const float cq = qs[h * nb + r / kBlock];
            float m = -INFINITY;
            for (int64_t j = 0; j < S; ++j) {
                const int32_t acc = dot_i8<DC>(qr, ik + (h * S + j) * D, D);
                s[(size_t) j] = (float) acc * (cq * ks[h * nb + j / kBlock] * scale);
                m = std::max(m, s[(size_t) j]);
            }
            std::fill(o.begin(), o.end(), 0.0f);
            float l = 0.0f;
            for (int64_t j = 0; j < S; ++j) {
                const float p = std::exp(s[(size_t) j] - m);
                l += p;
                axpy<DC>(o.data(), half_round(p), vf.data() + j * D, D);
            }
            for (int64_t d = 0; d < D; ++d) out[i * D + d] = f32_to_f16(o[(size_t) d] / l);
        });
    }
}
}  // namespace

extern "C" void orc_sage_rows(const int8_t* iq, const int8_t* ik, const uint16_t* hv, const float* qs, const float* ks,
                              int64_t S, int64_t H, int64_t D, float scale, const int64_t* rows_h, const int64_t* rows_s,
                              int64_t n, uint16_t* out) {
    if (D == 128) sage_rows_impl<128>(iq, ik, hv, qs, ks, S, H, D, scale, rows_h, rows_s, n, out);
    else sage_rows_impl<0>(iq, ik, hv, qs, ks, S, H, D, scale, rows_h, rows_s, n, out);
}

extern "C" {

// ---- fp16 fused SDPA semantics (kernels/h3sycl.cpp:1464-1500, oneDNN graph) on selected (head, row) pairs -------------
// q, k, v in dt, token rows at `stride`; each value goes through half first (the reference copies q, k, v to half,
// kernels/h3sycl.cpp:1543-1552). score f32 = sum of half products; x scale (f32); softmax in f32; probs rounded to half;
// out = half(sum of probs * v in f32). out half bits [n, D].
void orc_sdpa_rows(const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D, int64_t stride,
                   const int64_t* rows_h, const int64_t* rows_s, int64_t n, uint16_t* out) {
    (void) H;
    const float scale = 1.0f / std::sqrt((float) D);
    const int nt = threads();
    std::vector<std::vector<float>> s_t((size_t) nt, std::vector<float>((size_t) S));
    std::vector<std::vector<float>> o_t((size_t) nt, std::vector<float>((size_t) D)), q_t(o_t), k_t(o_t);
    par_for(n, 1, [&](int64_t i, int t) {
        std::vector<float>& s = s_t[(size_t) t];
        std::vector<float>& o = o_t[(size_t) t];
        std::vector<float>& qr = q_t[(size_t) t];
        std::vector<float>& kr = k_t[(size_t) t];
        const int64_t h = rows_h[i], r = rows_s[i];
        for (int64_t d = 0; d < D; ++d) qr[(size_t) d] = half_round(load(q, dt, (size_t) (r * stride + h * D + d)));
        float m = -INFINITY;
        for (int64_t j = 0; j < S; ++j) {
            for (int64_t d = 0; d < D; ++d) kr[(size_t) d] = half_round(load(k, dt, (size_t) (j * stride + h * D + d)));
            float acc = 0.0f;
            for (int64_t d = 0; d < D; ++d) acc += qr[(size_t) d] * kr[(size_t) d];
            s[(size_t) j] = acc * scale;
            m = std::max(m, s[(size_t) j]);
        }
        float l = 0.0f;
        for (int64_t j = 0; j < S; ++j) { s[(size_t) j] = std::exp(s[(size_t) j] - m); l += s[(size_t) j]; }
        std::fill(o.begin(), o.end(), 0.0f);
        for (int64_t j = 0; j < S; ++j) {
            const float p = half_round(s[(size_t) j] / l);
            for (int64_t d = 0; d < D; ++d) o[(size_t) d] += p * half_round(load(v, dt, (size_t) (j * stride + h * D + d)));
        }
        for (int64_t d = 0; d < D; ++d) out[i * D + d] = f32_to_f16(o[(size_t) d]);
    });
}

// ---- the exact reference: softmax(q k^T / sqrt(D)) v in float64 on the inputs as given ---------------------------------
// The tolerance anchor (per-row cosine and max-abs error are measured against this). out float32 [n, D].
void orc_exact_rows(const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D, int64_t stride,
                    const int64_t* rows_h, const int64_t* rows_s, int64_t n, float* out) {
    (void) H;
    const double scale = (double) (1.0f / std::sqrt((float) D));
    const int nt = threads();
    std::vector<std::vector<double>> s_t((size_t) nt, std::vector<double>((size_t) S));
    std::vector<std::vector<double>> o_t((size_t) nt, std::vector<double>((size_t) D)), q_t(o_t);
    par_for(n, 1, [&](int64_t i, int t) {
        std::vector<double>& s = s_t[(size_t) t];
        std::vector<double>& o = o_t[(size_t) t];
        std::vector<double>& qr = q_t[(size_t) t];
        const int64_t h = rows_h[i], r = rows_s[i];
        for (int64_t d = 0; d < D; ++d) qr[(size_t) d] = load(q, dt, (size_t) (r * stride + h * D + d));
        double m = -INFINITY;
        for (int64_t j = 0; j < S; ++j) {
            double acc = 0.0;
            for (int64_t d = 0; d < D; ++d) acc += qr[(size_t) d] * (double) load(k, dt, (size_t) (j * stride + h * D + d));
            s[(size_t) j] = acc * scale;
            m = std::max(m, s[(size_t) j]);
        }
        double l = 0.0;
        std::fill(o.begin(), o.end(), 0.0);
        for (int64_t j = 0; j < S; ++j) {
            const double p = std::exp(s[(size_t) j] - m);
            l += p;
            for (int64_t d = 0; d < D; ++d) o[(size_t) d] += p * (double) load(v, dt, (size_t) (j * stride + h * D + d));
        }
        for (int64_t d = 0; d < D; ++d) out[i * D + d] = (float) (o[(size_t) d] / l);
    });
}

// ---- h3s_attention as a whole (kernels/h3sycl.cpp:1779-1798), token-major out in out_dt ------------------------------
// sage_min_s: the Sage threshold (8192 by default in the reference); out [S, H*D] in out_dt. Returns 0, or -1 when the
// row stride is shorter than a row. The Sage path needs D in {64, 128} (kernels/sage.cpp:33).
int orc_attention(const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D, int64_t stride,
                  void* out, int out_dt, int64_t sage_min_s) {
    if (S <= 0 || H <= 0 || D <= 0) return 0;
    if (stride < H * D) return -1;
    const int64_t n = H * S;
    std::vector<int64_t> rh((size_t) n), rs((size_t) n);
    for (int64_t h = 0; h < H; ++h)
        for (int64_t s = 0; s < S; ++s) { rh[(size_t) (h * S + s)] = h; rs[(size_t) (h * S + s)] = s; }
    std::vector<uint16_t> ao((size_t) (n * D));
    if (S >= sage_min_s && (D == 64 || D == 128)) {
        const int64_t nb = (S + kBlock - 1) / kBlock;
        std::vector<int8_t> iq((size_t) (n * D)), ik((size_t) (n * D));
        std::vector<float> sc((size_t) (2 * H * nb + H * D));
        std::vector<uint16_t> hv((size_t) (n * D));
        orc_sage_prepass(q, k, v, dt, S, H, D, stride, iq.data(), ik.data(), sc.data(), hv.data());
        orc_sage_rows(iq.data(), ik.data(), hv.data(), sc.data(), sc.data() + H * nb, S, H, D, 1.0f / std::sqrt((float) D),
                      rh.data(), rs.data(), n, ao.data());
    } else {
        orc_sdpa_rows(q, k, v, dt, S, H, D, stride, rh.data(), rs.data(), n, ao.data());
    }
    // [H, S, D] half -> [S, H*D] out_dt through float (kernels/h3sycl.cpp:1769-1771)
    for (int64_t s = 0; s < S; ++s)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t d = 0; d < D; ++d)
                store(out, out_dt, (size_t) ((s * H + h) * D + d), f16_to_f32(ao[(size_t) ((h * S + s) * D + d)]));
    return 0;
}

// ---- per-head RMS norm + rotary rotation, in place (kernels/h3sycl.cpp:1276-1376; kernels/h3sycl.h:165-174) -------
// x: M token rows of H heads x D features at element stride `stride`, type dt; weight [D]; cs [M, rot_dim/2, 2].
// Returns 0, or -1 for the reference's refusals (rot_dim odd, above D, or leaving an odd remainder; stride < H*D).
// rsqrt is correctly rounded (the reference's sycl::rsqrt has implementation-defined accuracy).
int orc_rms_rope(void* x, int dt, int64_t M, int64_t H, int64_t D, int64_t stride, const float* weight, float eps,
                 const float* cs, int rot_dim) {
    if (M <= 0 || H <= 0 || D <= 0) return 0;
    if (rot_dim < 0 || rot_dim > D || rot_dim % 2 != 0 || (D - rot_dim) % 2 != 0) return -1;
    if (stride < H * D) return -1;
    const int64_t half = rot_dim / 2;
    par_for(M * H, 256, [&](int64_t mh, int) {
        const int64_t m = mh / H, h = mh % H;
        const size_t base = (size_t) (m * stride + h * D);
        float s = 0.0f;
        for (int64_t i = 0; i < D; ++i) {
            const float v = load(x, dt, base + (size_t) i);
            s += v * v;
        }
        const float arg = s / (float) D + eps;
        // 1/sqrt(arg) rounded once to float: the double result is within an ulp; the midpoints to its float
        // neighbours decide (r > mid  <=>  mid^2 * arg < 1, in long double, exact to far below any float tie)
        float y = (float) (1.0 / std::sqrt((double) arg));
        if (std::isfinite(y) && y > 0.0f && arg > 0.0f) {
            const float up = std::nextafter(y, INFINITY), dn = std::nextafter(y, 0.0f);
            const long double mu = ((long double) y + up) / 2, md = ((long double) y + dn) / 2;
            if (mu * mu * arg < 1.0L) y = up;
            else if (md * md * arg > 1.0L) y = dn;
        }
        const float inv = y;
        for (int64_t j = 0; j < half; ++j) {
            const size_t ia = base + (size_t) j, ib = base + (size_t) (half + j);
            const float a = load(x, dt, ia) * inv * weight[j];
            const float b = load(x, dt, ib) * inv * weight[half + j];
            const size_t t = (size_t) (m * half + j);
            const float co = cs[2 * t], si = cs[2 * t + 1];
            store(x, dt, ia, a * co - b * si);
            store(x, dt, ib, b * co + a * si);
        }
        for (int64_t i = rot_dim; i < D; ++i)
            store(x, dt, base + (size_t) i, load(x, dt, base + (size_t) i) * inv * weight[i]);
    });
    return 0;
}

// ---- causal attention with grouped heads (kernels/h3sycl.cpp:870-898; kernels/h3sycl.h:105-108) --------------------
// q rows of stride qs, k and v rows of stride kvs (elements), type dt; out [L, Hq*D] in dt. Query head h reads
// key/value head h / (Hq/Hkv). Every value is fp32 between the loads and the store (the reference never rounds P).
// The dot product is summed in feature order here (the reference's work-group reduction leaves its order open).
// Returns 0, or -1 for the reference's refusals (D > 256, Hq not a multiple of Hkv).
int orc_attention_causal(const void* q, const void* k, const void* v, int dt, int64_t L, int64_t Hq, int64_t Hkv,
                         int64_t D, int64_t qs, int64_t kvs, void* out) {
    if (L <= 0) return 0;
    if (D > 256 || Hkv <= 0 || Hq % Hkv != 0) return -1;
    const float scale = 1.0f / std::sqrt((float) D);
    par_for(Hq * L, 16, [&](int64_t hi, int) {
        const int64_t h = hi / L, i = hi % L, g = h / (Hq / Hkv);
        float m = -INFINITY, l = 0.0f;
        std::vector<float> acc((size_t) D, 0.0f);
        for (int64_t j = 0; j <= i; ++j) {
            float dot = 0.0f;
            for (int64_t d = 0; d < D; ++d)
                dot += load(q, dt, (size_t) (i * qs + h * D + d)) * load(k, dt, (size_t) (j * kvs + g * D + d));
            const float sc = dot * scale;
            const float mn = std::fmax(m, sc);
            const float a = std::exp(m - mn), e = std::exp(sc - mn);
            for (int64_t d = 0; d < D; ++d)
                acc[(size_t) d] = acc[(size_t) d] * a + e * load(v, dt, (size_t) (j * kvs + g * D + d));
            l = l * a + e;
            m = mn;
        }
        for (int64_t d = 0; d < D; ++d) store(out, dt, (size_t) (i * Hq * D + h * D + d), acc[(size_t) d] / l);
    });
    return 0;
}

// ---- int8 ConvRot linear (kernels/h3sycl.cpp:404-652; engine/h3-core/src/reference.rs:37-82) ----------------------
// The rotation of one group of g features in place, digit by digit (base 4) of the feature index, low digit first, as
// the reference's fused kernel applies h4 for g = 256 (kernels/h3sycl.cpp:404-470): for the four values x_0..x_3 that
// differ only in one digit, y_c = t - 2*x_(3-c). The sum t is ((x_0 + x_1) + x_2) + x_3 for the two low digits (inside
// a lane that holds 16 consecutive features) and (x_0 + x_1) + (x_2 + x_3) for the higher ones (across lanes: lane c
// forms (x_c + x_(c^1)) + (x_(c^2) + x_(c^3)), the same sum for every c); then the normalisation, 1/2 per digit.
// g = 2 * 4^n (accepted by the reference, whose matrix builder, kernels/h3sycl.cpp:185-200, then gives the top digit
// only the values 0 and 1, where h4's corner [[1, 1], [1, 1]] applies): y_0 = y_1 = x_0 + x_1 for that digit.
static void rot_group(float* v, int g) {
    int digit = 0;
    for (int d = 1; d < g; d *= 4, ++digit) {
        const bool in_thread = digit < 2;
        if (4 * d > g) {
            for (int e0 = 0; e0 < g; ++e0) {
                if ((e0 / d) % 2 != 0) continue;
                const float s = v[e0] + v[e0 + d];
                v[e0] = s;
                v[e0 + d] = s;
            }
            continue;
        }
        for (int e0 = 0; e0 < g; ++e0) {
            if ((e0 / d) % 4 != 0) continue;
            const float x[4] = {v[e0], v[e0 + d], v[e0 + 2 * d], v[e0 + 3 * d]};
            float y[4];
            if (in_thread) {
                const float t = ((x[0] + x[1]) + x[2]) + x[3];
                for (int c = 0; c < 4; ++c) y[c] = t - 2.0f * x[3 - c];
            } else {
                for (int c = 0; c < 4; ++c) {
                    const float t = (x[c] + x[c ^ 1]) + (x[c ^ 2] + x[c ^ 3]);
                    y[c] = t - 2.0f * x[c ^ 3];
                }
            }
            for (int c = 0; c < 4; ++c) v[e0 + c * d] = y[c];
        }
    }
    float norm = 1.0f;
    for (int d = 1; d < g; d *= 4) norm *= 0.5f;
    for (int e = 0; e < g; ++e) v[e] = v[e] * norm;
}

// Rotation (group 0: none) and per-row quantisation of x [M, K] (row stride K): xq int8 [M, K], rs [M] row scales.
void orc_rotq(const void* x, int dt, int64_t M, int64_t K, int group, int8_t* xq, float* rs) {
    par_for(M, 16, [&](int64_t r, int) {
        std::vector<float> v((size_t) K);
        for (int64_t i = 0; i < K; ++i) v[(size_t) i] = load(x, dt, (size_t) (r * K + i));
        if (group > 0)
            for (int64_t g0 = 0; g0 < K; g0 += group) rot_group(v.data() + g0, group);
        float m = 0.0f;
        for (int64_t i = 0; i < K; ++i) m = std::fmax(m, std::fabs(v[(size_t) i]));
        const float scale = std::fmax(m / 127.0f, 1e-30f);
        rs[r] = scale;
        for (int64_t i = 0; i < K; ++i) {
            const float q = std::nearbyint(v[(size_t) i] / scale);     // round half to even (the default mode)
            xq[(size_t) (r * K + i)] = (int8_t) std::fmin(127.0f, std::fmax(-128.0f, q));
        }
    });
}

// The whole layer: rotation + quantisation as above, int32 products, then the reference's rescale (kernels/h3sycl.cpp
// :573-599): one weight scale is folded into the row scale first (rs * ws, :573), so out = (float) acc * (rs * ws);
// per-output scales multiply after the row scale, out = ((float) acc * rs) * ws[n]; the bias is added last; each step
// rounded to float32, the result rounded to out_dt.
void orc_int8_linear(const void* x, int dt, int64_t M, int64_t K, const int8_t* w, int64_t N, const float* wscale,
                     int64_t n_wscale, const float* bias, void* out, int out_dt, int group) {
    std::vector<int8_t> xq((size_t) (M * K));
    std::vector<float> rs((size_t) M);
    orc_rotq(x, dt, M, K, group, xq.data(), rs.data());
    par_for(M, 4, [&](int64_t r, int) {
        for (int64_t n = 0; n < N; ++n) {
            int32_t acc = 0;
            for (int64_t i = 0; i < K; ++i) acc += (int32_t) xq[(size_t) (r * K + i)] * (int32_t) w[(size_t) (n * K + i)];
            float y = n_wscale > 1 ? ((float) acc * rs[(size_t) r]) * wscale[n] : (float) acc * (rs[(size_t) r] * wscale[0]);
            if (bias) y = y + bias[n];
            store(out, out_dt, (size_t) (r * N + n), y);
        }
    });
}

// engine/h3-core/src/reference.rs:37-82 as written there: x float32, the rotation a dense product with the normalised
// regular Hadamard matrix (acc += x_i * H[i][j] in feature order), round half to even; out float32 [M, N]. Defined for
// groups that are powers of 4 (reference.rs:4-5): its norm 1/sqrt(g) is the library's 2^-digits only there.
void orc_int8_linear_dense(const float* x, int64_t M, int64_t K, const int8_t* w, int64_t N, const float* wscale,
                           int64_t n_wscale, const float* bias, int group, float* out) {
    std::vector<float> h;
    if (group > 0) {
        static const int h4[4][4] = {{1, 1, 1, -1}, {1, 1, -1, 1}, {1, -1, 1, 1}, {-1, 1, 1, 1}};
        const float norm = 1.0f / std::sqrt((float) group);
        h.resize((size_t) group * group);
        for (int i = 0; i < group; ++i)
            for (int j = 0; j < group; ++j) {
                int sign = 1;
                for (int a = i, b = j, st = 1; st < group; st *= 4, a /= 4, b /= 4) sign *= h4[a % 4][b % 4];
                h[(size_t) i * group + j] = (float) sign * norm;
            }
    }
    par_for(M, 4, [&](int64_t r, int) {
        std::vector<float> xr((size_t) K);
        const float* row = x + r * K;
        if (group > 0) {
            for (int64_t g0 = 0; g0 < K; g0 += group)
                for (int j = 0; j < group; ++j) {
                    float acc = 0.0f;
                    for (int i = 0; i < group; ++i) acc += row[g0 + i] * h[(size_t) i * group + j];
                    xr[(size_t) (g0 + j)] = acc;
                }
        } else {
            for (int64_t i = 0; i < K; ++i) xr[(size_t) i] = row[i];
        }
        float m = 0.0f;
        for (float v : xr) m = std::fmax(m, std::fabs(v));
        const float scale = std::fmax(m / 127.0f, 1e-30f);
        std::vector<int32_t> q((size_t) K);
        for (int64_t i = 0; i < K; ++i) q[(size_t) i] = (int32_t) std::fmin(127.0f, std::fmax(-128.0f, std::nearbyint(xr[(size_t) i] / scale)));
        for (int64_t n = 0; n < N; ++n) {
            int32_t acc = 0;
            for (int64_t i = 0; i < K; ++i) acc += (int32_t) w[(size_t) (n * K + i)] * q[(size_t) i];
            const float ws = n_wscale == 1 ? wscale[0] : wscale[n];
            out[(size_t) (r * N + n)] = (float) acc * scale * ws + (bias ? bias[n] : 0.0f);
        }
    });
}

}  // extern "C"
