// h3sage.cu - libh3sage.so: SageAttention v1 for libh3cuda.so, the plugin interface of the reference's kernels/sage.cpp
// (maxfridbe/sycl_minimax_h3) on sm_100a. The kernel is attn_sage3 (attn3.cuh): int8 Q.K^T on tcgen05 kind::i8,
// dequantised with the per-block scales, online softmax, P.V in half on kind::f16, two 128-row query tiles per CTA.
//
// The reference's plugin wraps Intel's ARK kernel (kernels/sage.cpp:51-52) and its g_err is a process global
// (kernels/sage.cpp:23); so is this one's.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/h3sage.h"
#include "attn3.cuh"

namespace {

std::string g_err;
std::mutex g_mu;
constexpr int kMaxDevices = 64;
int* g_word[kMaxDevices] = {};          // the plugin's own error word per device (h3sage_check reads it)
constexpr uint64_t kDefaultWaitNs = 2000000000ull;

int fail(const std::string& m) {
    std::lock_guard<std::mutex> l(g_mu);
    g_err = m;
    return -1;
}

int* own_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> l(g_mu);
    if (!g_word[dev]) {
        int* w = nullptr;
        if (cudaMalloc(&w, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(w, 0, sizeof(int)) != cudaSuccess) { cudaFree(w); return nullptr; }
        g_word[dev] = w;
    }
    return g_word[dev];
}

// out_peers (P entries, P <= 8, S a multiple of P): the output rows of token s go to out_peers[s / (S / P)] at row
// s % (S / P) instead of to out (Ulysses groups; see h3sage_attention_peers)
int run(cudaStream_t st, const int8_t* q, const int8_t* k, const void* v, int64_t v_tok, int64_t v_head, void* out,
        int out_dt, int64_t out_tok, int64_t out_head, const float* qscale, const float* kscale, int block, int64_t S,
        int64_t H, int64_t D, float scale, int* err, uint64_t wait_ns, void* const* out_peers = nullptr, int P = 0) {
    if (D != 64 && D != 128) return fail("h3sage: head size " + std::to_string(D) + " (64 or 128)");
    if (block <= 0 || block % 64 != 0) return fail("h3sage: the scale block must be a multiple of 64");
    if (S <= 0 || H <= 0 || S > INT32_MAX / D / H) return fail("h3sage: sequence out of range");
    if (out_dt < 0 || out_dt > 2) return fail("h3sage: unknown output type " + std::to_string(out_dt));
    if (!err) err = own_word();
    if (!err) return fail("h3sage: no device error word (" + std::string(cudaGetErrorString(cudaGetLastError())) + ")");
    CUtensorMap mq, mk, mv;
    std::string e = h3::make_rows_map(&mq, q, true, D, S, H, 1, D, S * D, H * S * D, 0);
    if (e.empty()) e = h3::make_rows_map(&mk, k, true, D, S, H, 1, D, S * D, H * S * D, 0);
    // v: token-major (head stride the smaller) or packed by head
    const int v_order = v_head < v_tok ? 1 : 0;
    if (e.empty()) e = h3::make_rows_map(&mv, v, false, D, S, H, 1, v_tok * 2, v_head * 2, 0, v_order);
    if (!e.empty()) return fail("h3sage: " + e);
    h3::AttnArgs a{};
    a.S = (int) S;
    a.H = (int) H;
    a.n_kv = (int) ((S + h3::kTileN - 1) / h3::kTileN);
    a.scale_log2 = scale * 1.4426950408889634f;
    a.qs = qscale;
    a.ks = kscale;
    a.blk = block;
    a.nb = (int) ((S + block - 1) / block);
    a.out = out;
    a.out_seq = 0;
    a.out_tok = out_tok;
    a.out_head = out_head;
    a.out_dt = out_dt;
    const int es = out_dt == 0 ? 4 : 2;
    a.out_vec = ((reinterpret_cast<uintptr_t>(out) & 15) == 0 && (out_tok * es) % 16 == 0 && (out_head * es) % 16 == 0) ? 1 : 0;
    if (out_peers) {
        if (P < 1 || P > 8 || S % P != 0) return fail("h3sage: 1 to 8 ranks dividing the sequence");
        a.out_rows = (int) (S / P);
        for (int p = 0; p < P; ++p) {
            if (!out_peers[p]) return fail("h3sage: destination " + std::to_string(p) + " is null");
            a.out_peer[p] = out_peers[p];
            if (reinterpret_cast<uintptr_t>(out_peers[p]) & 15) a.out_vec = 0;
        }
    }
    a.q_order = 0;
    a.k_order = 0;
    a.v_order = v_order;
    a.err = err;
    a.wait_ns = wait_ns ? wait_ns : kDefaultWaitNs;
    a.D = (int) D;
    const cudaError_t ce = h3::launch_sage(mq, mk, mv, a, st);
    if (ce != cudaSuccess) return fail(std::string("h3sage: launch: ") + cudaGetErrorString(ce));
    return 0;
}

}  // namespace

extern "C" {

const char* h3sage_error(void) {
    std::lock_guard<std::mutex> l(g_mu);
    static thread_local std::string copy;
    copy = g_err;
    return copy.c_str();
}

int h3sage_attention(void* stream, const int8_t* q, const int8_t* k, const void* v, void* out, const float* qscale,
                     const float* kscale, int block, int64_t S, int64_t H, int64_t D, float scale) {
    cudaStream_t st = stream ? *static_cast<cudaStream_t*>(stream) : nullptr;
    // the plugin ABI's layouts: v and out half [H, S, D]
    return run(st, q, k, v, D, S * D, out, 1, D, S * D, qscale, kscale, block, S, H, D, scale, nullptr, 0);
}

int h3sage_attention_strided(void* stream, const int8_t* q, const int8_t* k, const void* v, int64_t v_tok, int64_t v_head,
                             void* out, int out_dt, int64_t out_tok, int64_t out_head, const float* qscale,
                             const float* kscale, int block, int64_t S, int64_t H, int64_t D, float scale, int* err,
                             uint64_t wait_ns) {
    cudaStream_t st = stream ? *static_cast<cudaStream_t*>(stream) : nullptr;
    return run(st, q, k, v, v_tok, v_head, out, out_dt, out_tok, out_head, qscale, kscale, block, S, H, D, scale, err,
               wait_ns);
}

int h3sage_attention_peers(void* stream, const int8_t* q, const int8_t* k, const void* v, int64_t v_tok, int64_t v_head,
                           void* const* out_peers, int P, int out_dt, int64_t out_tok, int64_t out_head,
                           const float* qscale, const float* kscale, int block, int64_t S, int64_t H, int64_t D,
                           float scale, int* err, uint64_t wait_ns) {
    cudaStream_t st = stream ? *static_cast<cudaStream_t*>(stream) : nullptr;
    if (!out_peers) return fail("h3sage: no destination table");
    return run(st, q, k, v, v_tok, v_head, out_peers[0], out_dt, out_tok, out_head, qscale, kscale, block, S, H, D,
               scale, err, wait_ns, out_peers, P);
}

int h3sage_check(void* stream) {
    cudaStream_t st = stream ? *static_cast<cudaStream_t*>(stream) : nullptr;
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(std::string("h3sage: ") + cudaGetErrorString(e));
    int* w = own_word();
    if (!w) return fail("h3sage: no device error word");
    int code = 0;
    e = cudaMemcpy(&code, w, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(std::string("h3sage: ") + cudaGetErrorString(e));
    if (code) {
        cudaMemset(w, 0, sizeof(int));
        return fail("h3sage: a wait inside the attention kernel gave up (code " + std::to_string(code) + ")");
    }
    return 0;
}

}  // extern "C"
