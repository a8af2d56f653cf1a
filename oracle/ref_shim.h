// ref_shim.h - a host-only stand-in for the few SYCL names that the reference's attention pre-pass, its dtype helpers
// and its RMS norm + RoPE use (kernels/h3sycl.cpp:38-63, 1276-1376, 1733-1771 of maxfridbe/sycl_minimax_h3), so that
// those lines compile unchanged with g++ and run on the CPU.
//
// TEST INFRASTRUCTURE ONLY (the checker). oracle/ref_build.py cuts the lines out of the reference's source into
// oracle/_ref/ at build time; nothing of the reference is stored in this repository.
//
// Semantics kept: a kernel runs every work-item of its range (OpenMP over independent items or work-groups; items of
// one group run in order); queue order is program order. sycl::fmax / fabs / round / clamp / min are the C library's
// (OpenCL's definitions: round half away from zero). sycl::half is _Float16 (conversions round to nearest even).
// reduce_over_group is the one collective: a work-group runs twice, first up to the reduction to collect every item's
// operand (the items do nothing else before it in these kernels), then in full with the reduced value.
// sycl::rsqrt has implementation-defined accuracy in SYCL; here it is correctly rounded (through double).
#pragma once
#include <omp.h>

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace sycl {

using half = _Float16;

template <class To, class From>
inline To bit_cast(const From& f) {
    static_assert(sizeof(To) == sizeof(From), "bit_cast of different sizes");
    To t;
    std::memcpy(&t, &f, sizeof(To));
    return t;
}

inline float fmax(float a, float b) { return std::fmax(a, b); }
inline float fabs(float x) { return std::fabs(x); }
inline float round(float x) { return std::round(x); }
inline float clamp(float x, float lo, float hi) { return std::fmin(std::fmax(x, lo), hi); }
inline float rsqrt(float x) { return (float) (1.0 / std::sqrt((double) x)); }
template <class T>
inline T min(T a, T b) { return b < a ? b : a; }

template <class T>
struct maximum {
    T operator()(const T& a, const T& b) const { return a < b ? b : a; }
};

template <int N>
struct range {
    size_t r[N];
    range(size_t a) : r{a} { static_assert(N == 1, "one extent"); }
    range(size_t a, size_t b) : r{a, b} { static_assert(N == 2, "two extents"); }
    range(size_t a, size_t b, size_t c) : r{a, b, c} { static_assert(N == 3, "three extents"); }
};

template <int N>
struct id {
    size_t v[N];
    size_t operator[](int i) const { return v[i]; }
};

template <int N>
struct nd_range {
    size_t global, local;
    nd_range(size_t g, size_t l) : global(g), local(l) { static_assert(N == 1, "1-D only"); }
    nd_range(range<1> g, range<1> l) : global(g.r[0]), local(l.r[0]) { static_assert(N == 1, "1-D only"); }
};

// One work-group's reduction state: the collecting pass records the operand and stops the item there.
struct group {
    std::vector<float>* collect;
    float value;
};
struct stop_at_reduction {};

template <int N>
struct nd_item {
    size_t grp, lid;
    group* g;
    size_t get_group(int) const { return grp; }
    size_t get_local_id(int) const { return lid; }
    group& get_group() const { return *g; }
};

inline float reduce_over_group(group& g, float x, maximum<float>) {
    if (g.collect) {
        g.collect->push_back(x);
        throw stop_at_reduction{};
    }
    return g.value;
}

template <class T, int N>
struct vec {
    T e[N];
    T& operator[](int i) { return e[i]; }
    const T& operator[](int i) const { return e[i]; }
};

struct queue {
    template <class F>
    void parallel_for(range<1> r, F f) {
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long) r.r[0]; ++i) f(id<1>{{(size_t) i}});
    }
    template <class F>
    void parallel_for(range<2> r, F f) {
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long) r.r[0]; ++i)
            for (size_t j = 0; j < r.r[1]; ++j) f(id<2>{{(size_t) i, j}});
    }
    template <class F>
    void parallel_for(range<3> r, F f) {
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long) r.r[0]; ++i)
            for (size_t j = 0; j < r.r[1]; ++j)
                for (size_t k = 0; k < r.r[2]; ++k) f(id<3>{{(size_t) i, j, k}});
    }
    template <class F>
    void parallel_for(nd_range<1> r, F f) {
        const long long groups = (long long) (r.global / r.local);
#pragma omp parallel for schedule(dynamic, 4)
        for (long long gi = 0; gi < groups; ++gi) {
            std::vector<float> ops;
            group g{&ops, 0.0f};
            bool reduces = false;
            for (size_t l = 0; l < r.local; ++l) {
                try {
                    f(nd_item<1>{(size_t) gi, l, &g});
                } catch (stop_at_reduction&) {
                    reduces = true;
                }
            }
            if (!reduces) continue;   // no reduction: every item already ran in full
            float m = ops[0];
            for (size_t i = 1; i < ops.size(); ++i) m = maximum<float>()(m, ops[i]);
            g.collect = nullptr;
            g.value = m;
            for (size_t l = 0; l < r.local; ++l) f(nd_item<1>{(size_t) gi, l, &g});
        }
    }
    void wait() {}
};

}  // namespace sycl
