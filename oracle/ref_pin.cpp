// ref_pin.cpp - the reference's own source for the attention pre-pass, its dtype helpers, its output relayout and
// h3s_rms_rope, compiled for the CPU (oracle/_ref/libref.so), to pin the oracle's restatement and the GPU kernels to
// the reference itself rather than to a reading of it.
//
// TEST INFRASTRUCTURE ONLY. The .inc files are cut out of the reference's kernels/h3sycl.cpp by oracle/ref_build.py
// into oracle/_ref/ (not part of this repository); this file supplies what surrounds them there:
//   h3sycl_dtype.inc     kernels/h3sycl.cpp:38-63    element types, bf16 conversions, load / store
//   h3sycl_rms_rope.inc  kernels/h3sycl.cpp:1276-1376 h3s_rms_rope (its scratch through the Ctx below)
//   h3sycl_prepass.inc   kernels/h3sycl.cpp:1733-1764 K mean, q / k quantiser, v to half [H, S, D]
//   h3sycl_out.inc       kernels/h3sycl.cpp:1769-1771 half [H, S, D] output to out_dt token rows
// The SYCL names they use come from ref_shim.h. The variables the pre-pass lines expect are set up as the enclosing
// function of the reference sets them (nb and the scale-buffer layout, kernels/h3sycl.cpp:1709,1716-1718).
#include "ref_shim.h"

namespace refsrc {

constexpr int kSageBlock = 64;   // kernels/h3sycl.cpp:1681

#include "h3sycl_dtype.inc"

// the part of the reference's context that h3s_rms_rope touches: its queue and one grow-only float buffer
struct Ctx {
    sycl::queue q;
    float* inv = nullptr;
    size_t inv_cap = 0;
    template <class T>
    T* grow(T*& p, size_t& cap, size_t n) {
        if (n <= cap) return p;
        std::free(p);
        p = static_cast<T*>(std::malloc(n * sizeof(T)));
        cap = p ? n : 0;
        if (!p) g_err = "ref: out of host memory";
        return p;
    }
    ~Ctx() { std::free(inv); }
};

#include "h3sycl_rms_rope.inc"

}  // namespace refsrc

extern "C" {

float ref_load(const void* p, int dt, uint64_t i) { return refsrc::load(p, dt, (size_t) i); }
void ref_store(void* p, int dt, uint64_t i, float v) { refsrc::store(p, dt, (size_t) i, v); }

// q, k, v: token rows of element stride `stride` in element type dt. Writes iq, ik int8 [H, S, D]; sc = q scales
// [H, nb], k scales [H, nb], k mean [H*D]; hv half bits [H, S, D].
void ref_sage_prepass(const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D,
                      int64_t stride, int8_t* iq, int8_t* ik, float* sc, uint16_t* hv) {
    using namespace refsrc;
    sycl::queue qu;
    const int64_t nb = (S + kSageBlock - 1) / kSageBlock;
    float* qs = sc;
    float* ks = sc + H * nb;
    float* kmean = sc + 2 * H * nb;
#include "h3sycl_prepass.inc"
}

// ao: half bits [H, S, D] -> out: out_dt [S, H*D]
void ref_out_relayout(const uint16_t* ao_bits, void* out, int out_dt, int64_t S, int64_t H, int64_t D) {
    using namespace refsrc;
    sycl::queue qu;
    const sycl::half* ao = reinterpret_cast<const sycl::half*>(ao_bits);
#include "h3sycl_out.inc"
}

int ref_rms_rope(void* x, int x_dt, int64_t M, int64_t H, int64_t D, int64_t stride, const float* weight, float eps,
                 const float* cs, int rot_dim) {
    refsrc::Ctx c;
    return refsrc::h3s_rms_rope(&c, x, x_dt, M, H, D, stride, weight, eps, cs, rot_dim);
}

const char* ref_error(void) { return refsrc::g_err.c_str(); }

}  // extern "C"
