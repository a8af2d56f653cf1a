// h3cuda.cu - libh3cuda.so: the attention subset of the reference's libh3sycl C ABI (kernels/h3sycl.h of
// maxfridbe/sycl_minimax_h3) on NVIDIA B200, sm_100a.
//
//   context + memory    kernels/h3sycl.cpp:77-174, 241-402: a CUDA stream per context (the in-order queue), counted
//                       allocations under a cap, grow-only scratch, pinned uploads on a second stream, per-thread errors
//   dispatcher          kernels/h3sycl.cpp:1779-1816: Sage when S >= sage_min_s and libh3sage.so loads, else fp16 SDPA
//   Sage pre-pass       kernels/h3sycl.cpp:1704-1764: K channel mean || Q quantiser, then K quantiser (prepass.cuh)
//   plugin loader       kernels/h3sycl.cpp:1683-1701: dlopen libh3sage.so from this library's directory
//   fp16 SDPA           kernels/h3sycl.cpp:1464-1674 (oneDNN's fused graph): attn_sage3<false> (attn3.cuh), reading
//                       q, k, v in place through TMA and writing the token-major output directly (no relayout copies)
//
// There is no CPU path and no score-table ("split") form: every attention call runs the tcgen05 kernels, or fails.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/h3cuda.h"
#include "../../include/h3sage.h"
#include "attn_common.cuh"
#include "prepass.cuh"
#include "attn3.cuh"
#include "rmsrope.cuh"
#include "causal.cuh"
#include "int8lin.cuh"
#include "ulysses.cuh"

namespace {

using namespace h3;

thread_local std::string g_err;
constexpr int kSageBlock = 64;   // kernels/h3sycl.cpp:1681

struct DeviceGuard {            // makes `dev` current for the call and restores the caller's device after
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int now = -1;
        if (prev >= 0 && cudaGetDevice(&now) == cudaSuccess && now != prev) cudaSetDevice(prev);
    }
};

struct Ctx {
    int device = 0;
    cudaStream_t st = nullptr;
    bool own_stream = false;
    cudaStream_t aux = nullptr;                  // the K mean beside the Q quantiser
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    cudaStream_t cs = nullptr;                   // uploads (h3s_upload), made on first use
    std::mutex cs_mu;
    std::string name;
    int* err = nullptr;                          // device error word of this context's kernels
    bool profile = false, poison = false;
    bool sage_want = true;
    int64_t sage_min_s = 8192;
    uint64_t wait_ns = 2000000000ull;
    int sage_state = 0;                          // 0 not loaded yet, 1 ready, -1 unavailable
    decltype(&h3sage_attention) sage_fn = nullptr;
    decltype(&h3sage_attention_strided) sage_strided = nullptr;
    decltype(&h3sage_attention_peers) sage_peers = nullptr;
    decltype(&h3sage_error) sage_err = nullptr;
    // scratch, grow-only
    int8_t* sq = nullptr; size_t sq_cap = 0;     // q, k as int8 [H, S, D]
    int8_t* sk = nullptr; size_t sk_cap = 0;
    float* ss = nullptr; size_t ss_cap = 0;      // q scales, k scales, k mean
    __half* hq = nullptr; size_t hq_cap = 0;     // half copies when the inputs cannot be read in place
    __half* hk = nullptr; size_t hk_cap = 0;
    __half* hv = nullptr; size_t hv_cap = 0;
    __half* ao = nullptr; size_t ao_cap = 0;     // [H, S, D] output of a plugin without the strided entry
    int8_t* lq = nullptr; size_t lq_cap = 0;     // int8 linear: quantised activations [rows, Kp]
    float* lrs = nullptr; size_t lrs_cap = 0;    //   their row scales
    int8_t* lw = nullptr; size_t lw_cap = 0;     //   the weight with rows padded to 16 bytes (K % 16 != 0 only)
    int n_sm = 148;
    std::mutex mem_mu;
    std::unordered_map<void*, size_t> mem;
    size_t mem_used = 0, mem_cap = 0;

    // A scratch buffer of at least n elements (+1/8 slack), counted against the cap; NULL with the reason in g_err.
    template <typename T> T* grow(T*& p, size_t& cap, size_t n) {
        if (n <= cap) return p;
        const size_t want = n + (n >> 3);
        std::lock_guard<std::mutex> l(mem_mu);
        if (mem_used - cap * sizeof(T) + want * sizeof(T) > mem_cap) {
            g_err = "a scratch buffer of " + std::to_string((want * sizeof(T)) >> 20) + " MiB would pass the device memory cap (" +
                    std::to_string(mem_used >> 20) + " of " + std::to_string(mem_cap >> 20) + " MiB in use)";
            return nullptr;
        }
        if (p) { cudaStreamSynchronize(st); cudaFree(p); }
        mem_used -= cap * sizeof(T);
        p = nullptr;
        if (cudaMalloc(&p, want * sizeof(T)) != cudaSuccess) { p = nullptr; cudaGetLastError(); }
        cap = p ? want : 0;
        mem_used += cap * sizeof(T);
        if (p && poison) cudaMemsetAsync(p, 0xff, want * sizeof(T), st);
        if (!p) g_err = "the device refused a scratch buffer of " + std::to_string((want * sizeof(T)) >> 20) + " MiB";
        return p;
    }
};

int cuda_fail(const char* what, cudaError_t e) {
    g_err = std::string(what) + ": " + cudaGetErrorString(e);
    return -1;
}

// The limit of every wait inside a kernel: H3S_WAIT_MS milliseconds, 2 s by default.
uint64_t env_wait_ns() {
    if (const char* e = std::getenv("H3S_WAIT_MS")) return (uint64_t) std::max(1, std::atoi(e)) * 1000000ull;
    return 2000000000ull;
}

// what every way of making a context shares (kernels/h3sycl.cpp:216-235)
bool init(Ctx& c) {
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, c.device) != cudaSuccess) { g_err = "cudaGetDeviceProperties failed"; return false; }
    c.name = p.name;
    c.n_sm = p.multiProcessorCount;
    double frac = 0.94;
    if (const char* e = std::getenv("H3S_MEM_FRACTION")) frac = std::min(0.97, std::max(0.05, std::atof(e)));
    c.mem_cap = (size_t) ((double) p.totalGlobalMem * frac);
    c.profile = std::getenv("H3S_PROFILE") != nullptr;
    c.poison = std::getenv("H3S_POISON") != nullptr;
    if (const char* e = std::getenv("H3S_ATTN")) c.sage_want = std::strcmp(e, "onednn") != 0 && std::strcmp(e, "sdpa") != 0;
    if (const char* e = std::getenv("H3S_SAGE_MIN_S")) c.sage_min_s = std::max<int64_t>(0, std::atoll(e));
    c.wait_ns = env_wait_ns();
    cudaError_t e;
    // the K mean (a few dozen CTAs, each a chain of S dependent adds: the pre-pass's critical path) runs on a stream of
    // the highest priority, so that its CTAs get SMs before the quantisers' thousands of CTAs queued beside it
    int prio_low = 0, prio_high = 0;
    cudaDeviceGetStreamPriorityRange(&prio_low, &prio_high);
    if ((e = cudaStreamCreateWithPriority(&c.aux, cudaStreamNonBlocking, prio_high)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&c.ev_fork, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&c.ev_join, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaMalloc(&c.err, sizeof(int))) != cudaSuccess || (e = cudaMemset(c.err, 0, sizeof(int))) != cudaSuccess) {
        cuda_fail("context", e);
        return false;
    }
    return true;
}

Ctx* make_ctx(int device, cudaStream_t st, bool own) {
    DeviceGuard g(device);
    auto* c = new Ctx;
    c->device = device;
    if (own) {
        cudaError_t e = cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking);
        if (e != cudaSuccess) { cuda_fail("cudaStreamCreate", e); delete c; return nullptr; }
        c->own_stream = true;
    } else {
        c->st = st;
    }
    if (!init(*c)) {
        if (c->own_stream) cudaStreamDestroy(c->st);
        delete c;
        return nullptr;
    }
    return c;
}

// ---- the Sage plugin (kernels/h3sycl.cpp:1683-1701) ----------------------------------------------------------------
std::mutex g_sage_mu;
bool sage_load(Ctx& c) {
    if (c.sage_state) return c.sage_state > 0;
    std::lock_guard<std::mutex> l(g_sage_mu);
    c.sage_state = -1;
    std::string path = "libh3sage.so";
    Dl_info me;
    if (dladdr((void*) &sage_load, &me) && me.dli_fname) {   // beside this library
        std::string self = me.dli_fname;
        const size_t slash = self.rfind('/');
        if (slash != std::string::npos) path = self.substr(0, slash + 1) + path;
    }
    void* h = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
    if (!h) { std::fprintf(stderr, "h3cuda: no SageAttention (%s); attention on the fp16 SDPA kernel\n", dlerror()); return false; }
    c.sage_fn = (decltype(c.sage_fn)) dlsym(h, "h3sage_attention");
    c.sage_err = (decltype(c.sage_err)) dlsym(h, "h3sage_error");
    c.sage_strided = (decltype(c.sage_strided)) dlsym(h, "h3sage_attention_strided");
    c.sage_peers = (decltype(c.sage_peers)) dlsym(h, "h3sage_attention_peers");
    if (!c.sage_fn || !c.sage_err) {
        std::fprintf(stderr, "h3cuda: %s lacks h3sage_attention; attention stays on the fp16 SDPA kernel\n", path.c_str());
        return false;
    }
    c.sage_state = 1;
    return true;
}

// ---- phase timing (H3S_PROFILE) ------------------------------------------------------------------------------------
struct Phases {
    Ctx& c;
    cudaEvent_t ev[4] = {};
    int n = 0;
    explicit Phases(Ctx& cc) : c(cc) {
        if (!c.profile) return;
        for (auto& e : ev) cudaEventCreate(&e);
    }
    void mark() {
        if (c.profile && n < 4) cudaEventRecord(ev[n++], c.st);
    }
    void report(const char* what, int64_t S) {
        if (!c.profile || n < 2) return;
        cudaEventSynchronize(ev[n - 1]);
        float ms[3] = {0, 0, 0};
        for (int i = 1; i < n; ++i) cudaEventElapsedTime(&ms[i - 1], ev[i - 1], ev[i]);
        std::fprintf(stderr, "h3cuda: attention (%s) S=%lld: pre-pass %.3f ms, attention %.3f, out %.3f\n", what,
                     (long long) S, ms[0], ms[1], ms[2]);
    }
    ~Phases() {
        if (!c.profile) return;
        for (auto& e : ev) cudaEventDestroy(e);
    }
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
int esize(int dt) { return dt == F32 ? 4 : 2; }

// The step before the attention in a denoiser block (engine/h3-core/src/dit.rs:347-348): RMS norm + RoPE of q and k in
// place (h3s_rms_rope, kernels/h3sycl.cpp:1276-1376), with q's and k's norm weights.
struct RopeArgs {
    const float* wq;
    const float* wk;
    float eps;
    const float* cs;
    int rot;
};

// ---- the Sage pre-pass (kernels/h3sycl.cpp:1733-1761) --------------------------------------------------------------
// With rope: q and k are normalised and rotated in place by the rms_rope kernel, as two h3s_rms_rope calls would (the
// same bits): k first, since the K mean needs it, then q on the main stream while the K mean runs beside it (measured
// at configs[3]: 0.63 against 0.70 ms for the step with both rotations before the fork). (A single pass that normalises q inside its quantiser, saving one read
// of q, measured slower at configs[3]: its rotation is compute-bound and, running beside the K mean, slows the K mean's
// chains, the pre-pass's critical path; the quantiser that runs there now is memory-bound.)
template <int DT>
int prepass_dt(Ctx& c, const void* q, const void* k, int64_t S, int64_t H, int64_t D, int64_t stride, int8_t* iq, int8_t* ik,
               float* sc, const RopeArgs* rope = nullptr) {
    const int64_t nb = (S + kSageBlock - 1) / kSageBlock;
    float* qs = sc;
    float* ks = sc + H * nb;
    float* kmean = sc + 2 * H * nb;
    const int C = (int) (H * D);
    const int es = DtInfo<DT>::ES;
    cudaError_t e;
    if (rope && (e = launch_rms_rope<DT>(const_cast<void*>(k), S, (int) H, (int) D, stride, rope->wk, rope->eps,
                                         rope->cs, rope->rot, c.st)) != cudaSuccess)
        return cuda_fail("rms_rope k", e);
    // fork: the K mean runs on the aux stream beside q's rotation and the Q quantiser
    if ((e = cudaEventRecord(c.ev_fork, c.st)) != cudaSuccess) return cuda_fail("event", e);
    if ((e = cudaStreamWaitEvent(c.aux, c.ev_fork, 0)) != cudaSuccess) return cuda_fail("event", e);
    if ((e = launch_kmean<DT>(k, S, C, stride, kmean, c.err, c.wait_ns, c.aux)) != cudaSuccess) return cuda_fail("kmean", e);
    if ((e = cudaEventRecord(c.ev_join, c.aux)) != cudaSuccess) return cuda_fail("event", e);
    const dim3 grid((unsigned) nb, (unsigned) H);
    const bool vq = aligned16(q) && (stride * es) % 16 == 0 && (D * es) % 16 == 0;
    const bool vk = aligned16(k) && (stride * es) % 16 == 0 && (D * es) % 16 == 0;
    // one quantiser launch: 64-row blocks x heads, the head size a template argument (64 or 128)
    auto quant = [&](const void* src, const float* mean, int8_t* dst, float* scales, bool vec) {
        if (D == 64) {
            if (vec) quant_rows<DT, 64, true><<<grid, kQuantThreads, 0, c.st>>>(src, (int) S, stride, mean, dst, scales, (int) nb);
            else quant_rows<DT, 64, false><<<grid, kQuantThreads, 0, c.st>>>(src, (int) S, stride, mean, dst, scales, (int) nb);
        } else {
            if (vec) quant_rows<DT, 128, true><<<grid, kQuantThreads, 0, c.st>>>(src, (int) S, stride, mean, dst, scales, (int) nb);
            else quant_rows<DT, 128, false><<<grid, kQuantThreads, 0, c.st>>>(src, (int) S, stride, mean, dst, scales, (int) nb);
        }
        return cudaGetLastError();
    };
    if (rope && (e = launch_rms_rope<DT>(const_cast<void*>(q), S, (int) H, (int) D, stride, rope->wq, rope->eps,
                                         rope->cs, rope->rot, c.st)) != cudaSuccess)
        return cuda_fail("rms_rope q", e);
    if ((e = quant(q, nullptr, iq, qs, vq)) != cudaSuccess) return cuda_fail("quantise q", e);
    if ((e = cudaStreamWaitEvent(c.st, c.ev_join, 0)) != cudaSuccess) return cuda_fail("event", e);
    if ((e = quant(k, kmean, ik, ks, vk)) != cudaSuccess) return cuda_fail("quantise k", e);
    return 0;
}

int prepass(Ctx& c, const void* q, const void* k, int dt, int64_t S, int64_t H, int64_t D, int64_t stride, int8_t* iq,
            int8_t* ik, float* sc, const RopeArgs* rope = nullptr) {
    if (D != 64 && D != 128) { g_err = "the Sage pre-pass takes D = 64 or 128 (got " + std::to_string(D) + ")"; return -1; }
    switch (dt) {
        case F16: return prepass_dt<F16>(c, q, k, S, H, D, stride, iq, ik, sc, rope);
        case BF16: return prepass_dt<BF16>(c, q, k, S, H, D, stride, iq, ik, sc, rope);
        case F32: return prepass_dt<F32>(c, q, k, S, H, D, stride, iq, ik, sc, rope);
        default: g_err = "unknown element type " + std::to_string(dt); return -1;
    }
}

// any dt token rows -> half [H, S, D] for one sequence
int to_half(Ctx& c, const void* src, int dt, int64_t S, int64_t H, int64_t D, int64_t stride, __half* dst, int64_t Dp = 0) {
    const int blocks = 148 * 8;
    const int dp = (int) (Dp > 0 ? Dp : D);
    switch (dt) {
        case F16: to_half_hsd<F16><<<blocks, 256, 0, c.st>>>(src, (int) S, (int) H, (int) D, stride, dst, dp); break;
        case BF16: to_half_hsd<BF16><<<blocks, 256, 0, c.st>>>(src, (int) S, (int) H, (int) D, stride, dst, dp); break;
        default: to_half_hsd<F32><<<blocks, 256, 0, c.st>>>(src, (int) S, (int) H, (int) D, stride, dst, dp); break;
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("to half", e);
}

// half [H, S, D] -> out_dt [S, H*D] (kernels/h3sycl.cpp:1769-1771), for a plugin without the strided entry point
__global__ void hsd_to_rows(const __half* src, int S, int H, int D, void* out, int out_dt) {
    const size_t n = (size_t) S * H * D;
    for (size_t i = blockIdx.x * (size_t) blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) {
        const size_t d = i % D, hh = (i / D) % H, s = i / ((size_t) D * H);
        const float v = __half2float(src[(hh * S + s) * D + d]);
        if (out_dt == F16) reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
        else if (out_dt == BF16) reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
        else reinterpret_cast<float*>(out)[i] = v;
    }
}

// ---- Form 0: SageAttention v1 (kernels/h3sycl.cpp:1704-1777). 1 = not a shape this path takes. ----------------------
// Output rows spread over the ranks of a Ulysses group (h3s_attention_ulysses): P token shards, row stride tok
// elements, each base already at this rank's head columns.
struct OutPeers {
    void* const* p;
    int P;
    int64_t tok;
};

int attention_sage(Ctx& c, const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D,
                   int64_t stride, void* out, int out_dt, const OutPeers* peers = nullptr, const RopeArgs* rope = nullptr,
                   bool* rotated = nullptr) {
    if ((D != 64 && D != 128) || S > INT32_MAX / D / H) return 1;   // the plugin's bounds (kernels/sage.cpp:33-35)
    if (peers && !c.sage_peers) return 1;
    const size_t n = (size_t) S * H * D;
    const int64_t nb = (S + kSageBlock - 1) / kSageBlock;
    int8_t* iq = c.grow(c.sq, c.sq_cap, n);
    int8_t* ik = c.grow(c.sk, c.sk_cap, n);
    float* sc = c.grow(c.ss, c.ss_cap, (size_t) (2 * H * nb + H * D));
    if (!iq || !ik || !sc) return -1;
    Phases ph(c);
    ph.mark();
    if (prepass(c, q, k, dt, S, H, D, stride, iq, ik, sc, rope) != 0) return -1;
    if (rope && rotated) *rotated = true;
    // v in place when the kernel can read it (half, 16-byte aligned rows); else a half copy by head
    const void* vp = v;
    int64_t v_tok = stride, v_head = D;
    const bool v_inplace = dt == F16 && aligned16(v) && (stride * 2) % 16 == 0 && c.sage_strided;
    if (!v_inplace) {
        __half* hv = c.grow(c.hv, c.hv_cap, n);
        if (!hv || to_half(c, v, dt, S, H, D, stride, hv) != 0) return -1;
        vp = hv;
        v_tok = D;
        v_head = S * D;
    }
    ph.mark();
    cudaStream_t st = c.st;
    const float scale = 1.0f / std::sqrt((float) D);
    const float* qs = sc;
    const float* ks = sc + H * nb;
    if (peers) {
        if (c.sage_peers(&st, iq, ik, vp, v_tok, v_head, peers->p, peers->P, out_dt, peers->tok, D, qs, ks, kSageBlock, S,
                         H, D, scale, c.err, c.wait_ns) != 0) {
            g_err = c.sage_err();
            return -2;
        }
        ph.mark();
    } else if (c.sage_strided) {
        if (c.sage_strided(&st, iq, ik, vp, v_tok, v_head, out, out_dt, H * D, D, qs, ks, kSageBlock, S, H, D, scale, c.err,
                           c.wait_ns) != 0) {
            g_err = c.sage_err();
            return -2;
        }
        ph.mark();
    } else {
        __half* ao = c.grow(c.ao, c.ao_cap, n);
        if (!ao) return -1;
        if (c.sage_fn(&st, iq, ik, vp, ao, qs, ks, kSageBlock, S, H, D, scale) != 0) { g_err = c.sage_err(); return -2; }
        ph.mark();
        hsd_to_rows<<<148 * 8, 256, 0, c.st>>>(ao, (int) S, (int) H, (int) D, out, out_dt);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail("out relayout", e);
    }
    ph.mark();
    ph.report("sage", S);
    return 0;
}

// ---- Form 1: fp16 SDPA over B sequences (kernels/h3sycl.cpp:1464-1674) ------------------------------------------------
int attention_sdpa(Ctx& c, const void* q, const void* k, const void* v, int dt, int64_t B, int64_t S, int64_t H, int64_t D,
                   int64_t stride, void* out, int out_dt, const OutPeers* peers = nullptr) {
    // any head size up to the kernel's 128 features: a narrower head is described to TMA with its true width and
    // reads as zeros beyond it (kernels/h3sycl.cpp:1464-1573 takes any D; wider heads are refused on this build)
    if (D > kHeadDim) {
        g_err = "attention: head size " + std::to_string(D) + " (at most " + std::to_string(kHeadDim) + " on this build)";
        return -1;
    }
    if (S > INT32_MAX / 2 || B * H > 65535) { g_err = "attention: sequence or head count out of range"; return -1; }
    Phases ph(c);
    ph.mark();
    const bool inplace = dt == F16 && D % 8 == 0 && aligned16(q) && aligned16(k) && aligned16(v) && (stride * 2) % 16 == 0;
    const void *qp = q, *kp = k, *vp = v;
    int order = 1;
    int64_t tok = stride * 2, head = D * 2, seq = S * stride * 2;
    if (!inplace) {
        const int64_t Dp = (D + 7) / 8 * 8;          // 16-byte rows
        const size_t per = (size_t) S * H * Dp, n = (size_t) B * per;
        __half* hq = c.grow(c.hq, c.hq_cap, n);
        __half* hk = c.grow(c.hk, c.hk_cap, n);
        __half* hv = c.grow(c.hv, c.hv_cap, n);
        if (!hq || !hk || !hv) return -1;
        const size_t ei = (size_t) esize(dt);
        for (int64_t b = 0; b < B; ++b) {
            const size_t io = (size_t) (b * S * stride) * ei;
            if (to_half(c, (const char*) q + io, dt, S, H, D, stride, hq + b * per, Dp) ||
                to_half(c, (const char*) k + io, dt, S, H, D, stride, hk + b * per, Dp) ||
                to_half(c, (const char*) v + io, dt, S, H, D, stride, hv + b * per, Dp))
                return -1;
        }
        qp = hq; kp = hk; vp = hv;
        order = 0;
        tok = Dp * 2; head = S * Dp * 2; seq = H * S * Dp * 2;
    }
    ph.mark();
    CUtensorMap mq, mk, mv;
    std::string e = make_rows_map(&mq, qp, false, D, S, H, B, tok, head, seq, order);
    if (e.empty()) e = make_rows_map(&mk, kp, false, D, S, H, B, tok, head, seq, order);
    if (e.empty()) e = make_rows_map(&mv, vp, false, D, S, H, B, tok, head, seq, order);
    if (!e.empty()) { g_err = "attention: " + e; return -1; }
    AttnArgs a{};
    a.S = (int) S;
    a.H = (int) H;
    a.n_kv = (int) ((S + kTileN - 1) / kTileN);
    a.scale_log2 = (1.0f / std::sqrt((float) D)) * 1.4426950408889634f;
    a.out = out;
    a.out_seq = S * H * D;
    a.out_tok = H * D;
    a.out_head = D;
    a.out_dt = out_dt;
    // 16-byte stores when every 32-feature chunk of every row starts on 16 bytes
    a.out_vec = aligned16(out) && (D * esize(out_dt)) % 16 == 0 ? 1 : 0;
    if (peers) {   // B = 1
        a.out_rows = (int) (S / peers->P);
        a.out_tok = peers->tok;
        if ((peers->tok * esize(out_dt)) % 16 != 0) a.out_vec = 0;
        for (int p = 0; p < peers->P; ++p) {
            a.out_peer[p] = peers->p[p];
            if (!aligned16(peers->p[p])) a.out_vec = 0;
        }
        a.out = peers->p[0];
    }
    a.q_order = a.k_order = a.v_order = order;
    a.err = c.err;
    a.wait_ns = c.wait_ns;
    a.D = (int) D;
    const cudaError_t ce = launch_sdpa(mq, mk, mv, a, (int) B, c.st);
    if (ce != cudaSuccess) return cuda_fail("attention launch", ce);
    ph.mark();
    ph.mark();
    ph.report("sdpa", S);
    return 0;
}

int check_dt(int dt) { return dt == F32 || dt == F16 || dt == BF16; }

// the wait self-test: an mbarrier nothing arrives at
__global__ void wait_timeout_kernel(int* err, unsigned long long wait_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !mbar_wait(&bar, 0, wait_ns, nullptr)) atomicOr(err, 16);
    __syncthreads();
}

// ---- the allocation-free Sage path (h3s_attention_sage_static) -------------------------------------------------------
// For callers that cannot allocate device memory when they call: code on a path that must not synchronise the device
// (cudaMalloc / cudaFree may), and hosts whose device memory is wholly owned and budgeted by another allocator. Its
// scratch (the int8 q and k and their scales) lives in this fixed array instead, which every GPU that loads this
// library holds until the process exits. Each GPU has its own copy; calls on one GPU share it, so overlapping calls
// race. The first call on a device looks the address up (cudaGetSymbolAddress), before any stream capture.
constexpr size_t kStaticMaxElems = size_t(4) << 20;           // S * H * D of one call, at most
constexpr size_t kStaticMaxHD = 16384;                          // H * D of one call, at most
constexpr size_t kStaticScaleBytes = 128 << 10;                 // q scales, k scales, k mean
constexpr size_t kStaticBytes = 2 * kStaticMaxElems + kStaticScaleBytes;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticBytes];

std::mutex g_static_mu;
uint8_t* g_static_ptr[64] = {};                                 // the array's device address, per device

// The device address of the scratch array on the current device (cudaGetSymbolAddress once per device).
uint8_t* static_scratch(int dev) {
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> l(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) { cuda_fail("cudaGetSymbolAddress", e); return nullptr; }
        g_static_ptr[dev] = static_cast<uint8_t*>(p);
    }
    return g_static_ptr[dev];
}

// h3s_rms_rope's refusals (kernels/h3sycl.cpp:1279-1283)
bool check_rope(const char* who, int64_t D, int rot_dim) {
    if (rot_dim < 0 || rot_dim > D || rot_dim % 2 != 0 || (D - rot_dim) % 2 != 0) {
        g_err = std::string(who) + ": rot_dim must be even, at most D, and leave an even remainder";
        return false;
    }
    return true;
}

}  // namespace

extern "C" {

const char* h3s_last_error(void) { return g_err.c_str(); }

void* h3s_open(void) { return h3s_open_gpu(0); }

int h3s_gpu_count(void) {
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail("cudaGetDeviceCount", e);
    return n;
}

int h3s_gpu_info(int index, char* name, int name_len, uint64_t* mem_bytes, char* pci, int pci_len) {
    const int n = h3s_gpu_count();
    if (n < 0) return -1;
    if (index < 0 || index >= n) { g_err = "no GPU " + std::to_string(index); return -1; }
    cudaDeviceProp p{};
    const cudaError_t e = cudaGetDeviceProperties(&p, index);
    if (e != cudaSuccess) return cuda_fail("cudaGetDeviceProperties", e);
    if (name && name_len > 0) std::snprintf(name, (size_t) name_len, "%s", p.name);
    if (mem_bytes) *mem_bytes = p.totalGlobalMem;
    if (pci && pci_len > 0) std::snprintf(pci, (size_t) pci_len, "%04x:%02x:%02x.0", p.pciDomainID, p.pciBusID, p.pciDeviceID);
    return 0;
}

void* h3s_open_gpu(int index) {
    const int n = h3s_gpu_count();
    if (n < 0) return nullptr;
    if (index < 0 || index >= n) {
        g_err = "no GPU " + std::to_string(index) + " (" + std::to_string(n) + " found)";
        return nullptr;
    }
    return make_ctx(index, nullptr, true);
}

void* h3s_create(void* stream) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { cuda_fail("cudaGetDevice", e); return nullptr; }
    return make_ctx(dev, stream ? *static_cast<cudaStream_t*>(stream) : nullptr, false);
}

void h3s_destroy(void* ctx) {
    auto* c = static_cast<Ctx*>(ctx);
    if (!c) return;
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->st);
    cudaStreamSynchronize(c->aux);
    if (c->cs) { cudaStreamSynchronize(c->cs); cudaStreamDestroy(c->cs); }
    for (void* p : {(void*) c->sq, (void*) c->sk, (void*) c->ss, (void*) c->hq, (void*) c->hk, (void*) c->hv, (void*) c->ao,
                    (void*) c->lq, (void*) c->lrs, (void*) c->lw, (void*) c->err})
        if (p) cudaFree(p);
    for (auto& kv : c->mem) cudaFree(kv.first);
    cudaEventDestroy(c->ev_fork);
    cudaEventDestroy(c->ev_join);
    cudaStreamDestroy(c->aux);
    if (c->own_stream) cudaStreamDestroy(c->st);
    delete c;
}

const char* h3s_device_name(void* ctx) { return static_cast<Ctx*>(ctx)->name.c_str(); }
uint64_t h3s_mem_cap(void* ctx) { return static_cast<Ctx*>(ctx)->mem_cap; }
uint64_t h3s_mem_used(void* ctx) {
    auto& c = *static_cast<Ctx*>(ctx);
    std::lock_guard<std::mutex> l(c.mem_mu);
    return c.mem_used;
}
uint64_t h3s_mem_free(void* ctx) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    size_t f = 0, t = 0;
    if (cudaMemGetInfo(&f, &t) != cudaSuccess) { cudaGetLastError(); return 0; }
    return f;
}

void* h3s_alloc(void* ctx, uint64_t bytes) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    std::lock_guard<std::mutex> l(c.mem_mu);
    if (c.mem_used + bytes > c.mem_cap) {
        g_err = "h3s_alloc: " + std::to_string(bytes >> 20) + " MiB would pass the device memory cap (" +
                std::to_string(c.mem_used >> 20) + " of " + std::to_string(c.mem_cap >> 20) + " MiB in use)";
        return nullptr;
    }
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes ? bytes : 1);
    if (e != cudaSuccess) {
        cudaGetLastError();
        g_err = "h3s_alloc: the device refused " + std::to_string(bytes >> 20) + " MiB (" + cudaGetErrorString(e) + ")";
        return nullptr;
    }
    if (c.poison) { cudaMemset(p, 0xff, bytes ? bytes : 1); }
    c.mem.emplace(p, bytes);
    c.mem_used += bytes;
    return p;
}

void h3s_free(void* ctx, void* p) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (!p) return;
    DeviceGuard g(c.device);
    cudaStreamSynchronize(c.st);                 // nothing queued may still read or write it
    if (c.cs) cudaStreamSynchronize(c.cs);       // nor an upload into it
    std::lock_guard<std::mutex> l(c.mem_mu);
    auto it = c.mem.find(p);
    if (it == c.mem.end()) return;
    c.mem_used -= it->second;
    c.mem.erase(it);
    cudaFree(p);
}

int h3s_write(void* ctx, void* dst, const void* src_host, uint64_t bytes) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    cudaError_t e = cudaMemcpyAsync(dst, src_host, bytes, cudaMemcpyHostToDevice, c.st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.st);
    return e == cudaSuccess ? 0 : cuda_fail("h3s_write", e);
}

int h3s_read(void* ctx, void* dst_host, const void* src, uint64_t bytes) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    cudaError_t e = cudaMemcpyAsync(dst_host, src, bytes, cudaMemcpyDeviceToHost, c.st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.st);
    return e == cudaSuccess ? 0 : cuda_fail("h3s_read", e);
}

int h3s_copy(void* ctx, void* dst, const void* src, uint64_t bytes) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, c.st);
    return e == cudaSuccess ? 0 : cuda_fail("h3s_copy", e);
}

int h3s_wait(void* ctx) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    cudaError_t e = cudaStreamSynchronize(c.st);
    if (e != cudaSuccess) return cuda_fail("h3s_wait", e);
    int code = 0;
    e = cudaMemcpy(&code, c.err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail("h3s_wait", e);
    if (code) {
        cudaMemset(c.err, 0, sizeof(int));
        g_err = "h3s_wait: a wait inside a kernel gave up after " + std::to_string(c.wait_ns / 1000000) +
                " ms (code " + std::to_string(code) + "); its results are not valid";
        return -1;
    }
    return 0;
}

void* h3s_alloc_host(void* ctx, uint64_t bytes) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    void* p = nullptr;
    const cudaError_t e = cudaMallocHost(&p, bytes ? bytes : 1);
    if (e != cudaSuccess) {
        cudaGetLastError();
        g_err = "h3s_alloc_host: the runtime refused " + std::to_string(bytes >> 20) + " MiB of pinned memory";
        return nullptr;
    }
    return p;
}

void h3s_free_host(void* ctx, void* p) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (!p) return;
    DeviceGuard g(c.device);
    if (c.cs) cudaStreamSynchronize(c.cs);
    cudaFreeHost(p);
}

int h3s_upload(void* ctx, void* dst, const void* src_pinned, uint64_t bytes) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    cudaPointerAttributes as{}, ad{};
    if (cudaPointerGetAttributes(&as, src_pinned) != cudaSuccess || cudaPointerGetAttributes(&ad, dst) != cudaSuccess ||
        as.type != cudaMemoryTypeHost || ad.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        g_err = "h3s_upload: the source must be h3s_alloc_host memory and the destination device memory";
        return -1;
    }
    {
        std::lock_guard<std::mutex> l(c.cs_mu);
        if (!c.cs) {
            const cudaError_t e = cudaStreamCreateWithFlags(&c.cs, cudaStreamNonBlocking);
            if (e != cudaSuccess) return cuda_fail("h3s_upload", e);
        }
    }
    const cudaError_t e = cudaMemcpyAsync(dst, src_pinned, bytes, cudaMemcpyHostToDevice, c.cs);
    return e == cudaSuccess ? 0 : cuda_fail("h3s_upload", e);
}

int h3s_upload_wait(void* ctx) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    if (!c.cs) return 0;
    const cudaError_t e = cudaStreamSynchronize(c.cs);
    return e == cudaSuccess ? 0 : cuda_fail("h3s_upload_wait", e);
}

int h3s_attention(void* ctx, const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D,
                  int64_t stride, void* out, int out_dt) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (S <= 0 || H <= 0 || D <= 0) return 0;
    if (stride < H * D) { g_err = "h3s_attention: the row stride is shorter than a row"; return -1; }
    if (!check_dt(dt) || !check_dt(out_dt)) { g_err = "h3s_attention: unknown element type"; return -1; }
    DeviceGuard g(c.device);
    if (c.sage_want && S >= c.sage_min_s && sage_load(c)) {
        const int rc = attention_sage(c, q, k, v, dt, S, H, D, stride, out, out_dt);
        if (rc == 0) return 0;
        if (rc == -1) return -1;
        if (rc == -2) {   // the plugin refused: as the reference, log, wait, and stay on the SDPA kernel from now on
            std::fprintf(stderr, "h3cuda: SageAttention failed (%s); attention stays on the fp16 SDPA kernel\n", g_err.c_str());
            cudaStreamSynchronize(c.st);
            c.sage_state = -1;
        }
    }
    return attention_sdpa(c, q, k, v, dt, 1, S, H, D, stride, out, out_dt);
}

int h3s_attention_batch(void* ctx, const void* q, const void* k, const void* v, int dt, int64_t B, int64_t S, int64_t H,
                        int64_t D, int64_t stride, void* out, int out_dt) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (B <= 0 || S <= 0 || H <= 0 || D <= 0) return 0;
    if (stride < H * D) { g_err = "h3s_attention_batch: the row stride is shorter than a row"; return -1; }
    if (!check_dt(dt) || !check_dt(out_dt)) { g_err = "h3s_attention_batch: unknown element type"; return -1; }
    const bool sage = c.sage_want && S >= c.sage_min_s;
    if (B > 1 && !sage) {
        DeviceGuard g(c.device);
        return attention_sdpa(c, q, k, v, dt, B, S, H, D, stride, out, out_dt);
    }
    const size_t ei = (size_t) esize(dt), eo = (size_t) esize(out_dt);
    for (int64_t b = 0; b < B; ++b) {
        const size_t io = (size_t) (b * S * stride) * ei, oo = (size_t) (b * S * H * D) * eo;
        const int rc = h3s_attention(ctx, (const char*) q + io, (const char*) k + io, (const char*) v + io, dt, S, H, D, stride,
                                     (char*) out + oo, out_dt);
        if (rc != 0) return rc;
    }
    return 0;
}

// h3s_attention for the heads of one rank of a Ulysses group, with the output rows stored straight into the token
// shards of every rank (include/h3cuda.h)
int h3s_attention_ulysses(void* ctx, const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H,
                          int64_t D, int64_t stride, void* const* out_shards, int P, int rank, int out_dt) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (S <= 0 || H <= 0 || D <= 0) return 0;
    if (stride < H * D) { g_err = "h3s_attention_ulysses: the row stride is shorter than a row"; return -1; }
    if (!check_dt(dt) || !check_dt(out_dt)) { g_err = "h3s_attention_ulysses: unknown element type"; return -1; }
    if (P < 1 || P > 8 || rank < 0 || rank >= P || S % P != 0 || !out_shards) {
        g_err = "h3s_attention_ulysses: 1 to 8 ranks dividing the sequence, and a destination per rank";
        return -1;
    }
    const size_t oe = out_dt == F32 ? 4 : 2;
    void* bases[8];
    for (int p = 0; p < P; ++p) {
        if (!out_shards[p]) { g_err = "h3s_attention_ulysses: destination " + std::to_string(p) + " is null"; return -1; }
        bases[p] = static_cast<char*>(out_shards[p]) + (size_t) rank * H * D * oe;
    }
    const OutPeers peers{bases, P, (int64_t) P * H * D};
    DeviceGuard g(c.device);
    if (c.sage_want && S >= c.sage_min_s && sage_load(c)) {
        const int rc = attention_sage(c, q, k, v, dt, S, H, D, stride, nullptr, out_dt, &peers);
        if (rc == 0) return 0;
        if (rc == -1) return -1;
        if (rc == -2) {
            std::fprintf(stderr, "h3cuda: SageAttention failed (%s); attention stays on the fp16 SDPA kernel\n", g_err.c_str());
            cudaStreamSynchronize(c.st);
            c.sage_state = -1;
        }
    }
    return attention_sdpa(c, q, k, v, dt, 1, S, H, D, stride, nullptr, out_dt, &peers);
}

// kernels/h3sycl.cpp:870-898: the reference's refusals (D <= 256, Hq a multiple of Hkv), the arithmetic in causal.cuh
int h3s_attention_causal(void* ctx, const void* q, const void* k, const void* v, int dt, int64_t L, int64_t Hq,
                         int64_t Hkv, int64_t D, int64_t qs, int64_t kvs, void* out) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (L <= 0) return 0;
    if (D <= 0 || D > 256 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) {
        g_err = "h3s_attention_causal: D <= 256, Hq a multiple of Hkv";
        return -1;
    }
    if (qs < Hq * D || kvs < Hkv * D) { g_err = "h3s_attention_causal: a row stride is shorter than its heads"; return -1; }
    if (!check_dt(dt)) { g_err = "h3s_attention_causal: unknown element type " + std::to_string(dt); return -1; }
    if (L > INT32_MAX / Hq) { g_err = "h3s_attention_causal: too many rows"; return -1; }
    DeviceGuard g(c.device);
    cudaError_t e;
    switch (dt) {
        case F16: e = launch_causal<F16>(q, k, v, (int) L, (int) Hq, (int) Hkv, (int) D, qs, kvs, out, c.st); break;
        case BF16: e = launch_causal<BF16>(q, k, v, (int) L, (int) Hq, (int) Hkv, (int) D, qs, kvs, out, c.st); break;
        default: e = launch_causal<F32>(q, k, v, (int) L, (int) Hq, (int) Hkv, (int) D, qs, kvs, out, c.st); break;
    }
    return e == cudaSuccess ? 0 : cuda_fail("h3s_attention_causal", e);
}

// kernels/h3sycl.cpp:1276-1376: the reference's refusals and degenerate sizes, the arithmetic in rmsrope.cuh
int h3s_rms_rope(void* ctx, void* x, int x_dt, int64_t M, int64_t H, int64_t D, int64_t stride, const float* weight,
                 float eps, const float* cs, int rot_dim) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (M <= 0 || H <= 0 || D <= 0) return 0;
    if (rot_dim < 0 || rot_dim > D || rot_dim % 2 != 0 || (D - rot_dim) % 2 != 0) {
        g_err = "h3s_rms_rope: rot_dim must be even, at most D, and leave an even remainder";
        return -1;
    }
    if (stride < H * D) { g_err = "h3s_rms_rope: the row stride is shorter than a row"; return -1; }
    if (!check_dt(x_dt)) { g_err = "h3s_rms_rope: unknown element type " + std::to_string(x_dt); return -1; }
    if (M * H > (int64_t) INT32_MAX * kRopeRows) { g_err = "h3s_rms_rope: too many rows"; return -1; }
    DeviceGuard g(c.device);
    cudaError_t e;
    switch (x_dt) {
        case F16: e = launch_rms_rope<F16>(x, M, (int) H, (int) D, stride, weight, eps, cs, rot_dim, c.st); break;
        case BF16: e = launch_rms_rope<BF16>(x, M, (int) H, (int) D, stride, weight, eps, cs, rot_dim, c.st); break;
        default: e = launch_rms_rope<F32>(x, M, (int) H, (int) D, stride, weight, eps, cs, rot_dim, c.st); break;
    }
    return e == cudaSuccess ? 0 : cuda_fail("h3s_rms_rope", e);
}

// kernels/h3sycl.cpp:632-652 (the entry point, its refusals and row chunks) and :404-630 (the layer), the arithmetic in
// int8lin.cuh. Row chunks bound the int8 copy of the activations at 1 GiB.
int h3s_int8_linear(void* ctx, const void* x, int x_dt, int64_t M, int64_t K, const int8_t* w, int64_t N,
                    const float* wscale, int64_t n_wscale, const float* bias, void* out, int out_dt, int group) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (M <= 0 || K <= 0 || N <= 0) return 0;
    if (group > 0 && (group > 256 || K % group != 0 || (group & (group - 1)) != 0)) {
        g_err = "h3s_int8_linear: unsupported ConvRot group size";
        return -1;
    }
    if (!check_dt(x_dt) || !check_dt(out_dt)) { g_err = "h3s_int8_linear: unknown element type"; return -1; }
    if (n_wscale < 1 || (n_wscale > 1 && n_wscale < N)) {
        g_err = "h3s_int8_linear: n_wscale must be 1 or N";
        return -1;
    }
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX - 16) { g_err = "h3s_int8_linear: too large"; return -1; }
    DeviceGuard g(c.device);
    const int64_t Kp = (K + 15) / 16 * 16;
    const int64_t rows_max = std::max<int64_t>(kLinBM, ((int64_t) 1 << 30) / Kp / kLinBM * kLinBM);
    const int64_t n_nb = (N + kLinBN - 1) / kLinBN;
    // the tile count of a chunk stays an int: rows x column blocks <= 2^30 tiles
    const int64_t rows_tiles = std::max<int64_t>(kLinBM, ((int64_t) 1 << 30) / n_nb * kLinBM);
    const int64_t R = std::min({M, rows_max, rows_tiles});
    int8_t* xq = c.grow(c.lq, c.lq_cap, (size_t) (R * Kp));
    float* rs = c.grow(c.lrs, c.lrs_cap, (size_t) R);
    if (!xq || !rs) return -1;
    cudaError_t e;
    const int8_t* wk = w;
    if (K != Kp || (reinterpret_cast<uintptr_t>(w) & 15)) {
        int8_t* wp = c.grow(c.lw, c.lw_cap, (size_t) (N * Kp));
        if (!wp) return -1;
        pad_rows_i8<<<c.n_sm * 4, 256, 0, c.st>>>(w, (int) N, (int) K, (int) Kp, wp);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("h3s_int8_linear", e);
        wk = wp;
    }
    CUtensorMap tb;
    std::string why = make_i8_map(&tb, wk, Kp, N, Kp, lin_weight_rows());
    if (!why.empty()) { g_err = "h3s_int8_linear: weight map: " + why; return -1; }
    LinArgs a{};
    a.N = (int) N;
    a.nkb = (int) ((Kp + kLinBK - 1) / kLinBK);
    a.n_nb = (int) n_nb;
    // a band of column blocks whose slice of W (256 rows x Kp bytes each) takes at most 64 MiB of L2
    a.band = (int) std::max<int64_t>(1, std::min<int64_t>(a.n_nb, ((int64_t) 64 << 20) / (kLinBN * Kp)));
    a.rs = rs;
    a.ws = wscale;
    a.per_n = n_wscale > 1;
    a.bias = bias;
    a.out_dt = out_dt;
    a.err = c.err;
    a.wait_ns = c.wait_ns;
    const size_t xe = x_dt == F32 ? 4 : 2, oe = out_dt == F32 ? 4 : 2;
    for (int64_t r0 = 0; r0 < M; r0 += R) {
        const int rows = (int) std::min(R, M - r0);
        const void* xr = static_cast<const char*>(x) + (size_t) r0 * K * xe;
        switch (x_dt) {
            case F16: e = launch_rotq<F16>(xr, rows, (int) K, (int) Kp, group, xq, rs, c.n_sm, c.st); break;
            case BF16: e = launch_rotq<BF16>(xr, rows, (int) K, (int) Kp, group, xq, rs, c.n_sm, c.st); break;
            default: e = launch_rotq<F32>(xr, rows, (int) K, (int) Kp, group, xq, rs, c.n_sm, c.st); break;
        }
        if (e != cudaSuccess) return cuda_fail("h3s_int8_linear", e);
        CUtensorMap ta;
        why = make_i8_map(&ta, xq, Kp, rows, Kp, kLinBM);
        if (!why.empty()) { g_err = "h3s_int8_linear: activation map: " + why; return -1; }
        a.M = rows;
        a.n_mb = (rows + lin_rows_per_tile() - 1) / lin_rows_per_tile();
        a.out = static_cast<char*>(out) + (size_t) r0 * N * oe;
        a.out_vec = (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && ((size_t) N * oe) % 16 == 0;
        if ((e = launch_i8gemm(ta, tb, a, c.n_sm, c.st)) != cudaSuccess) return cuda_fail("h3s_int8_linear", e);
    }
    return 0;
}

// ---- the Ulysses exchange over peer memory (ulysses.cuh) ------------------------------------------------------------
int h3s_ipc_handle(void* ctx, const void* ptr, void* handle) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (!ptr || !handle) { g_err = "h3s_ipc_handle: null pointer"; return -1; }
    DeviceGuard g(c.device);
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) return cuda_fail("h3s_ipc_handle", e);
    static_assert(sizeof(h) == 64, "a CUDA IPC handle is 64 bytes");
    std::memcpy(handle, &h, sizeof(h));
    return 0;
}

void* h3s_ipc_open(void* ctx, const void* handle) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (!handle) { g_err = "h3s_ipc_open: null handle"; return nullptr; }
    DeviceGuard g(c.device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) { cuda_fail("h3s_ipc_open", e); return nullptr; }
    return p;
}

int h3s_ipc_close(void* ctx, void* ptr) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (!ptr) return 0;
    DeviceGuard g(c.device);
    cudaStreamSynchronize(c.st);
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? 0 : cuda_fail("h3s_ipc_close", e);
}

// the checks both directions share; fills the peer table
static int ulysses_args(const char* what, int64_t s, int64_t H, int64_t D, int es, int P, int rank, void* const* dst,
                        PeerBases& pb) {
    if (P < 1 || P > kMaxPeers || rank < 0 || rank >= P) { g_err = std::string(what) + ": 1 to 8 ranks"; return -1; }
    if (s <= 0 || H <= 0 || D <= 0 || H % P != 0 || (es != 2 && es != 4)) {
        g_err = std::string(what) + ": s, H, D > 0, H a multiple of the ranks, 2- or 4-byte elements";
        return -1;
    }
    if (!dst) { g_err = std::string(what) + ": no destination table"; return -1; }
    for (int p = 0; p < kMaxPeers; ++p) pb.p[p] = p < P ? static_cast<char*>(dst[p]) : nullptr;
    for (int p = 0; p < P; ++p)
        if (!pb.p[p]) { g_err = std::string(what) + ": destination " + std::to_string(p) + " is null"; return -1; }
    return 0;
}

int h3s_ulysses_push_qkv(void* ctx, const void* shard, int64_t s, int64_t H, int64_t D, int es, int P, int rank,
                         void* const* dst) {
    auto& c = *static_cast<Ctx*>(ctx);
    PeerBases pb;
    if (ulysses_args("h3s_ulysses_push_qkv", s, H, D, es, P, rank, dst, pb) != 0) return -1;
    if (!shard) { g_err = "h3s_ulysses_push_qkv: null shard"; return -1; }
    DeviceGuard g(c.device);
    const cudaError_t e = launch_push_qkv(shard, s, (int) H, (int) D, es, P, rank, pb, c.n_sm, c.st);
    return e == cudaSuccess ? 0 : cuda_fail("h3s_ulysses_push_qkv", e);
}

int h3s_ulysses_push_out(void* ctx, const void* out_heads, int64_t s, int64_t H, int64_t D, int es, int P, int rank,
                         void* const* dst) {
    auto& c = *static_cast<Ctx*>(ctx);
    PeerBases pb;
    if (ulysses_args("h3s_ulysses_push_out", s, H, D, es, P, rank, dst, pb) != 0) return -1;
    if (!out_heads) { g_err = "h3s_ulysses_push_out: null output"; return -1; }
    DeviceGuard g(c.device);
    const cudaError_t e = launch_push_out(out_heads, s, (int) H, (int) D, es, P, rank, pb, c.n_sm, c.st);
    return e == cudaSuccess ? 0 : cuda_fail("h3s_ulysses_push_out", e);
}

int h3s_sage_prepass(void* ctx, const void* q, const void* k, int dt, int64_t S, int64_t H, int64_t D, int64_t stride,
                     int8_t* iq, int8_t* ik, float* sc) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (S <= 0 || H <= 0 || D <= 0) return 0;
    if (stride < H * D) { g_err = "h3s_sage_prepass: the row stride is shorter than a row"; return -1; }
    if (!check_dt(dt)) { g_err = "h3s_sage_prepass: unknown element type"; return -1; }
    DeviceGuard g(c.device);
    return prepass(c, q, k, dt, S, H, D, stride, iq, ik, sc);
}

// h3s_rms_rope on q and on k, then h3s_sage_prepass, with q's normalisation fused into its quantiser's pass
// (include/h3cuda.h)
int h3s_sage_prepass_rope(void* ctx, void* q, void* k, int dt, int64_t S, int64_t H, int64_t D, int64_t stride,
                          const float* wq, const float* wk, float eps, const float* cs, int rot_dim, int8_t* iq,
                          int8_t* ik, float* sc) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (S <= 0 || H <= 0 || D <= 0) return 0;
    if (!check_rope("h3s_sage_prepass_rope", D, rot_dim)) return -1;
    if (stride < H * D) { g_err = "h3s_sage_prepass_rope: the row stride is shorter than a row"; return -1; }
    if (!check_dt(dt)) { g_err = "h3s_sage_prepass_rope: unknown element type"; return -1; }
    DeviceGuard g(c.device);
    const RopeArgs rope{wq, wk, eps, cs, rot_dim};
    return prepass(c, q, k, dt, S, H, D, stride, iq, ik, sc, &rope);
}

// The attention half of a denoiser block's step before its output projection (engine/h3-core/src/dit.rs:347-350):
// h3s_rms_rope(q), h3s_rms_rope(k), h3s_attention, in one call (include/h3cuda.h)
int h3s_attention_rms_rope(void* ctx, void* q, void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D,
                           int64_t stride, void* out, int out_dt, const float* wq, const float* wk, float eps,
                           const float* cs, int rot_dim) {
    auto& c = *static_cast<Ctx*>(ctx);
    if (S <= 0 || H <= 0 || D <= 0) return 0;
    if (!check_rope("h3s_attention_rms_rope", D, rot_dim)) return -1;
    if (stride < H * D) { g_err = "h3s_attention_rms_rope: the row stride is shorter than a row"; return -1; }
    if (!check_dt(dt) || !check_dt(out_dt)) { g_err = "h3s_attention_rms_rope: unknown element type"; return -1; }
    DeviceGuard g(c.device);
    const RopeArgs rope{wq, wk, eps, cs, rot_dim};
    bool rotated = false;
    if (c.sage_want && S >= c.sage_min_s && sage_load(c)) {
        const int rc = attention_sage(c, q, k, v, dt, S, H, D, stride, out, out_dt, nullptr, &rope, &rotated);
        if (rc == 0) return 0;
        if (rc == -1) return -1;
        if (rc == -2) {   // as h3s_attention: log, wait, stay on the SDPA kernel from now on
            std::fprintf(stderr, "h3cuda: SageAttention failed (%s); attention stays on the fp16 SDPA kernel\n", g_err.c_str());
            cudaStreamSynchronize(c.st);
            c.sage_state = -1;
        }
    }
    if (!rotated) {   // the SDPA path reads q and k as they are: normalise and rotate them first (once)
        if (h3s_rms_rope(ctx, q, dt, S, H, D, stride, wq, eps, cs, rot_dim) != 0) return -1;
        if (h3s_rms_rope(ctx, k, dt, S, H, D, stride, wk, eps, cs, rot_dim) != 0) return -1;
    }
    return attention_sdpa(c, q, k, v, dt, 1, S, H, D, stride, out, out_dt);
}

void* h3s_stream(void* ctx) { return (void*) static_cast<Ctx*>(ctx)->st; }

int h3s_selftest_wait_timeout(void* ctx, uint64_t wait_ns) {
    auto& c = *static_cast<Ctx*>(ctx);
    DeviceGuard g(c.device);
    wait_timeout_kernel<<<1, 32, 0, c.st>>>(c.err, (unsigned long long) wait_ns);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail("h3s_selftest_wait_timeout", e);
}

int h3s_attention_sage_static(void* stream, const void* q, const void* k, const void* v, int64_t S, int64_t H, int64_t D,
                              int64_t stride, void* out, int out_dt, int* err) {
    if (S <= 0 || H <= 0 || D <= 0) return 0;
    if (D != 128) { g_err = "h3s_attention_sage_static: head size " + std::to_string(D) + " (128 only)"; return -1; }
    if (stride < H * D) { g_err = "h3s_attention_sage_static: the row stride is shorter than a row"; return -1; }
    if ((size_t) S * H * D > kStaticMaxElems || (size_t) (H * D) > kStaticMaxHD) {
        g_err = "h3s_attention_sage_static: S*H*D = " + std::to_string(S * H * D) + ", H*D = " + std::to_string(H * D) +
                " is beyond the fixed scratch (S*H*D <= " + std::to_string(kStaticMaxElems) + ", H*D <= " +
                std::to_string(kStaticMaxHD) + ")";
        return -1;
    }
    if (!check_dt(out_dt)) { g_err = "h3s_attention_sage_static: unknown output type"; return -1; }
    if (!err) { g_err = "h3s_attention_sage_static: err must be a device int of the caller"; return -1; }
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (stride * 2) % 16 != 0) {
        g_err = "h3s_attention_sage_static: q, k, v must start on 16 bytes and the row stride be a multiple of 8";
        return -1;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail("h3s_attention_sage_static", e);
    uint8_t* base = static_scratch(dev);
    if (!base) return -1;
    cudaStream_t st = stream ? *static_cast<cudaStream_t*>(stream) : nullptr;
    const int64_t nb = (S + kSageBlock - 1) / kSageBlock;    // H*nb <= S*H/64 + H <= 640: the scales fit 128 KiB
    int8_t* iq = reinterpret_cast<int8_t*>(base);
    int8_t* ik = reinterpret_cast<int8_t*>(base + kStaticMaxElems);
    float* sc = reinterpret_cast<float*>(base + 2 * kStaticMaxElems);
    float* qs = sc;
    float* ks = sc + H * nb;
    float* kmean = sc + 2 * H * nb;
    const int C = (int) (H * D);
    // the caller's error word starts each call at zero (a set word makes the attention kernel skip its work)
    if ((e = cudaMemsetAsync(err, 0, sizeof(int), st)) != cudaSuccess) return cuda_fail("h3s_attention_sage_static", e);
    // K mean (one chain per channel), then the two quantisers, all on the caller's stream
    const uint64_t wait_ns = env_wait_ns();
    if ((e = launch_kmean<F16>(k, S, C, stride, kmean, err, wait_ns, st)) != cudaSuccess)
        return cuda_fail("h3s_attention_sage_static", e);
    const dim3 grid((unsigned) nb, (unsigned) H);
    quant_rows<F16, 128, true><<<grid, kQuantThreads, 0, st>>>(q, (int) S, stride, nullptr, iq, qs, (int) nb);
    quant_rows<F16, 128, true><<<grid, kQuantThreads, 0, st>>>(k, (int) S, stride, kmean, ik, ks, (int) nb);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("h3s_attention_sage_static", e);
    // the int8 attention, v read in place, out written in place
    CUtensorMap mq, mk, mv;
    std::string me = make_rows_map(&mq, iq, true, D, S, H, 1, D, S * D, H * S * D, 0);
    if (me.empty()) me = make_rows_map(&mk, ik, true, D, S, H, 1, D, S * D, H * S * D, 0);
    if (me.empty()) me = make_rows_map(&mv, v, false, D, S, H, 1, stride * 2, D * 2, 0, 1);
    if (!me.empty()) { g_err = "h3s_attention_sage_static: " + me; return -1; }
    AttnArgs a{};
    a.S = (int) S;
    a.H = (int) H;
    a.n_kv = (int) ((S + kTileN - 1) / kTileN);
    a.scale_log2 = (1.0f / std::sqrt((float) D)) * 1.4426950408889634f;
    a.qs = qs;
    a.ks = ks;
    a.nb = (int) nb;
    a.blk = kSageBlock;
    a.out = out;
    a.out_tok = H * D;
    a.out_head = D;
    a.out_dt = out_dt;
    a.out_vec = aligned16(out) ? 1 : 0;
    a.q_order = a.k_order = 0;
    a.v_order = 1;
    a.err = err;
    a.wait_ns = wait_ns;
    a.D = (int) D;
    if ((e = launch_sage(mq, mk, mv, a, st)) != cudaSuccess) return cuda_fail("h3s_attention_sage_static", e);
    return 0;
}

}  // extern "C"
