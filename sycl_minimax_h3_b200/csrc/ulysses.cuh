// ulysses.cuh - the Ulysses head <-> sequence exchange as stores into the other GPUs' memory (one process per GPU on
// one node, NVLink/NVSwitch): each rank writes the part of its data that another rank needs straight into that
// rank's buffer, in the layout that rank computes on. The relayout and the transfer are one pass; what is left of a
// collective is for the ranks to meet before they read what they received.
//
// Layouts (P ranks, this rank r, s = S/P token rows per rank, h = H/P heads per rank, D features, es bytes each):
//   shard     [s, 3*H*D]     this rank's token rows r*s .. r*s+s-1 of a qkv buffer (q | k | v, all heads)
//   heads     [P*s, 3*h*D]   every rank's buffer for the attention of its heads over all tokens (q | k | v)
//   out_heads [P*s, h*D]     this rank's attention output (its heads, all tokens)
//   out_shard [s, H*D]       every rank's token rows of the output, all heads
// push_qkv: shard[t, part, p*h + hl, :] -> heads_p[r*s + t, part, hl, :]
// push_out: out_heads[p*s + t, hl, :]  -> out_shard_p[t, r*h + hl, :]
// 16-byte vectors when every row and head segment is a multiple of 16 bytes and the bases are 16-byte aligned (the
// host checks), single elements otherwise. Plain stores to peer memory; no multicast.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace h3 {

constexpr int kMaxPeers = 8;
struct PeerBases {
    char* p[kMaxPeers];
};

template <int VB>   // bytes per copy unit: 16, or the element size
__global__ void u_push_qkv(const char* __restrict__ shard, long long s, int H, int D, int es, int P, int rank,
                           PeerBases dst) {
    const int h = H / P;
    const long long row_b = 3LL * H * D * es;                 // bytes of a shard row
    const long long units_row = row_b / VB;
    const long long total = s * units_row;
    const long long hrow_b = 3LL * h * D * es;                // bytes of a heads row
    const long long part_b = (long long) H * D * es, head_b = (long long) D * es;
    for (long long u = blockIdx.x * (long long) blockDim.x + threadIdx.x; u < total; u += (long long) gridDim.x * blockDim.x) {
        const long long t = u / units_row, cb = (u % units_row) * VB;   // byte column in the shard row
        const int part = (int) (cb / part_b);
        const long long wb = cb % part_b;
        const int head = (int) (wb / head_b);
        const long long db = wb % head_b;
        const int p = head / h, hl = head % h;
        char* d = dst.p[p] + ((long long) rank * s + t) * hrow_b + (long long) part * h * head_b + hl * head_b + db;
        const char* sp = shard + t * row_b + cb;
        if constexpr (VB == 16) *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(sp);
        else if constexpr (VB == 4) *reinterpret_cast<uint32_t*>(d) = *reinterpret_cast<const uint32_t*>(sp);
        else *reinterpret_cast<uint16_t*>(d) = *reinterpret_cast<const uint16_t*>(sp);
    }
}

template <int VB>
__global__ void u_push_out(const char* __restrict__ out_heads, long long s, int H, int D, int es, int P, int rank,
                           PeerBases dst) {
    const int h = H / P;
    const long long row_b = (long long) h * D * es;           // bytes of an out_heads row
    const long long units_row = row_b / VB;
    const long long total = (long long) P * s * units_row;
    const long long orow_b = (long long) H * D * es;          // bytes of an out_shard row
    for (long long u = blockIdx.x * (long long) blockDim.x + threadIdx.x; u < total; u += (long long) gridDim.x * blockDim.x) {
        const long long g = u / units_row, cb = (u % units_row) * VB;
        const int p = (int) (g / s);
        const long long t = g % s;
        char* d = dst.p[p] + t * orow_b + (long long) rank * row_b + cb;
        const char* sp = out_heads + g * row_b + cb;
        if constexpr (VB == 16) *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(sp);
        else if constexpr (VB == 4) *reinterpret_cast<uint32_t*>(d) = *reinterpret_cast<const uint32_t*>(sp);
        else *reinterpret_cast<uint16_t*>(d) = *reinterpret_cast<const uint16_t*>(sp);
    }
}

// the copy unit both kernels can use: 16 bytes when every segment and base allows it, else the element size
inline int u_unit(long long seg_bytes, int es, const void* src, const PeerBases& dst, int P) {
    bool v16 = seg_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
    for (int p = 0; p < P; ++p) v16 = v16 && (reinterpret_cast<uintptr_t>(dst.p[p]) & 15) == 0;
    return v16 ? 16 : es;
}

inline cudaError_t launch_push_qkv(const void* shard, long long s, int H, int D, int es, int P, int rank,
                                   const PeerBases& dst, int n_sm, cudaStream_t st) {
    const int unit = u_unit((long long) D * es, es, shard, dst, P);
    const char* src = static_cast<const char*>(shard);
    const unsigned grid = (unsigned) n_sm * 8;
    if (unit == 16) u_push_qkv<16><<<grid, 256, 0, st>>>(src, s, H, D, es, P, rank, dst);
    else if (unit == 4) u_push_qkv<4><<<grid, 256, 0, st>>>(src, s, H, D, es, P, rank, dst);
    else u_push_qkv<2><<<grid, 256, 0, st>>>(src, s, H, D, es, P, rank, dst);
    return cudaGetLastError();
}

inline cudaError_t launch_push_out(const void* out_heads, long long s, int H, int D, int es, int P, int rank,
                                   const PeerBases& dst, int n_sm, cudaStream_t st) {
    const int unit = u_unit((long long) (H / P) * D * es, es, out_heads, dst, P);
    const char* src = static_cast<const char*>(out_heads);
    const unsigned grid = (unsigned) n_sm * 8;
    if (unit == 16) u_push_out<16><<<grid, 256, 0, st>>>(src, s, H, D, es, P, rank, dst);
    else if (unit == 4) u_push_out<4><<<grid, 256, 0, st>>>(src, s, H, D, es, P, rank, dst);
    else u_push_out<2><<<grid, 256, 0, st>>>(src, s, H, D, es, P, rank, dst);
    return cudaGetLastError();
}

}  // namespace h3
