// attn_common.cuh - what the attention kernel (attn3.cuh) and its hosts share: the argument block, tile sizes,
// error bits, the softmax's int32 -> float trick, TMEM stores, the epilogue that writes output rows (rounded through
// half, then to the output type: kernels/h3sycl.cpp:1769-1771), and the TMA maps over token rows.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <string>

#include "ptx.cuh"

namespace h3 {

enum Dt : int { F32 = 0, F16 = 1, BF16 = 2 };

constexpr int kTileM = 128;   // query rows per CTA
constexpr int kTileN = 128;   // keys per K/V tile
constexpr int kHeadDim = 128;
constexpr uint32_t kTmemCols = 512;

// error word bits a kernel sets when one of its waits gave up
constexpr int kErrProducer = 1, kErrMma = 2, kErrSoftmax = 4, kErrPrepass = 8;

struct AttnArgs {
    int S;                      // tokens per sequence
    int H;                      // heads (grid.y = H * sequences)
    int n_kv;                   // key tiles, ceil(S / 128)
    float scale_log2;           // softmax scale * log2(e)
    const float* qs;            // int8 path: Q scales [H, nb], one per `blk` rows
    const float* ks;            // int8 path: K scales [H, nb]
    int nb, blk;
    void* out;                  // output element (b, s, h, d) at out + b*out_seq + s*out_tok + h*out_head + d
    long long out_seq, out_tok, out_head;
    int out_dt;                 // F16 / BF16 / F32; values go through half first (kernels/h3sycl.cpp:1769-1771)
    int out_vec;                // 16-byte stores allowed (alignment checked on the host)
    int q_order, k_order, v_order;   // 0: map dims (D, S, H, B); 1: map dims (D, H, S, B)
    int* err;                   // device error word
    unsigned long long wait_ns; // limit of every wait
    int D;                      // head size: the kernel runs 128 wide (64 wide for the fp16 path's heads up to 64),
                                // and a narrower head reads as zeros in the features past D (TMA fills what lies
                                // outside the tensor with zeros), so those features of Q.K^T add nothing and those of
                                // P.V come out 0 and are not stored
    // Output rows spread over the ranks of a Ulysses group (out_rows > 0): token s goes to out_peer[s / out_rows], a
    // rank's token shard in its own or another GPU's memory (base already at this rank's head columns), at row
    // s % out_rows; out is then unused. out_rows = 0: every row to out.
    int out_rows;
    void* out_peer[8];
};


__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void tma_rows(void* dst, const CUtensorMap* map, uint64_t* bar, int order, int c0, int row,
                                         int head, int seq) {
    if (order) tma_load_4d(dst, map, bar, c0, head, row, seq);
    else tma_load_4d(dst, map, bar, c0, row, head, seq);
}


// n <= 32 consecutive output features of one row (fp32 values already divided by the row sum), rounded to half,
// then to out_dt (kernels/h3sycl.cpp:1769-1771), stored at out + e0 elements (16-byte stores for whole chunks).
__device__ __forceinline__ void store_out32(const AttnArgs& a, void* out, long long e0, const float (&val)[32], int n) {
    __half hv[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) hv[i] = __float2half_rn(val[i]);
    const bool vec = a.out_vec && n == 32;
    if (a.out_dt == F16) {
        __half* dst = reinterpret_cast<__half*>(out) + e0;
        if (vec) {
#pragma unroll
            for (int v = 0; v < 4; ++v) reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(hv)[v];
        } else {
            for (int i = 0; i < n; ++i) dst[i] = hv[i];
        }
    } else if (a.out_dt == BF16) {
        __nv_bfloat16 bv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) bv[i] = __float2bfloat16_rn(__half2float(hv[i]));
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out) + e0;
        if (vec) {
#pragma unroll
            for (int v = 0; v < 4; ++v) reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(bv)[v];
        } else {
            for (int i = 0; i < n; ++i) dst[i] = bv[i];
        }
    } else {
        float fv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) fv[i] = __half2float(hv[i]);
        float* dst = reinterpret_cast<float*>(out) + e0;
        if (vec) {
#pragma unroll
            for (int v = 0; v < 8; ++v) reinterpret_cast<float4*>(dst)[v] = reinterpret_cast<const float4*>(fv)[v];
        } else {
            for (int i = 0; i < n; ++i) dst[i] = fv[i];
        }
    }
}

// The epilogue of one query row, features col0 .. col0 + 32*chunks - 1 (those below a.D): O (fp32, in TMEM columns
// from o_taddr, which holds feature col0) / l, stored at out + b*out_seq + qrow*out_tok + h*out_head + feature.
// Warp-collective (TMEM loads): every lane calls it; rows past S (live = false) load but do not store. With out_rows > 0
// (a Ulysses group) the row goes to its rank's token shard out_peer[qrow / out_rows] at row qrow % out_rows.
__device__ __forceinline__ void store_out_cols(const AttnArgs& a, int b, int h, int qrow, uint32_t o_taddr, float inv,
                                               bool live, int col0, int chunks) {
    void* out = a.out;
    int row = qrow;
    if (a.out_rows > 0 && live) {
        const int p = qrow / a.out_rows;
        row = qrow - p * a.out_rows;
        out = a.out_peer[p & 7];
    }
    const long long base = (long long) b * a.out_seq + (long long) row * a.out_tok + (long long) h * a.out_head + col0;
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
        if (c4 >= chunks || col0 + c4 * 32 >= a.D) break;
        uint32_t o[32];
        tmem_ld32(o_taddr + c4 * 32, o);
        tmem_wait_ld();
        if (!live) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]) * inv;
        store_out32(a, out, base + c4 * 32, v, min(32, a.D - col0 - c4 * 32));
    }
}
__device__ __forceinline__ void store_out_row(const AttnArgs& a, int b, int h, int qrow, uint32_t o_taddr, float inv, bool live) {
    store_out_cols(a, b, h, qrow, o_taddr, inv, live, 0, 4);
}

// The output rows of one warp through shared memory. A thread owns one query row, so direct 16-byte stores put 32
// rows' chunks in each warp store (32 cache lines per instruction); staged, each store instruction writes 512
// consecutive bytes of two rows.
constexpr int kStagePitch = 272;                  // 256 bytes of a row + 16: the 32 rows' 16-byte chunks in distinct banks
constexpr int kStageWarpBytes = 32 * kStagePitch;

// 32 O columns scaled by inv, rounded through half (kernels/h3sycl.cpp:1769-1771) and packed in the out type:
// 16 words for F16 / BF16, 32 for F32. Packed conversions (two values per instruction, each rounded to nearest even).
__device__ __forceinline__ void pack_out32(int out_dt, const uint32_t (&o)[32], float inv, uint32_t (&w)[32]) {
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        const __half2 h2 = __floats2half2_rn(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv);
        if (out_dt == F16) {
            w[i / 2] = *reinterpret_cast<const uint32_t*>(&h2);
        } else {
            const float2 f = __half22float2(h2);
            if (out_dt == BF16) {
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(f.x, f.y);
                w[i / 2] = *reinterpret_cast<const uint32_t*>(&b2);
            } else {
                w[i] = __float_as_uint(f.x);
                w[i + 1] = __float_as_uint(f.y);
            }
        }
    }
}

// Rows row0 .. row0+31 (this lane: row0 + lane) of O at o_taddr, times inv, to the output. stage: this warp's
// kStageWarpBytes of shared memory that nothing else uses any more. Needs a.out_vec (16-byte aligned rows whose byte
// length is a multiple of 16). Rows at or past S are not stored.
__device__ __forceinline__ void store_out_staged(const AttnArgs& a, int b, int h, int row0, int lane, uint32_t o_taddr,
                                                 float inv, uint8_t* stage) {
    const int esz = a.out_dt == F32 ? 4 : 2;
    const int cpp = 256 / esz;                         // columns per pass: 256 bytes of each row
    // this lane's row: its first byte in the output (null past S)
    uint8_t* dst = nullptr;
    {
        const int q = row0 + lane;
        if (q < a.S) {
            void* out = a.out;
            int row = q;
            if (a.out_rows > 0) {
                const int p = q / a.out_rows;
                row = q - p * a.out_rows;
                out = a.out_peer[p & 7];
            }
            dst = reinterpret_cast<uint8_t*>(out) +
                  ((long long) b * a.out_seq + (long long) row * a.out_tok + (long long) h * a.out_head) * esz;
        }
    }
    fence_proxy_async_smem();                          // the stage held TMA-written, MMA-read tiles
    for (int col0 = 0; col0 < a.D; col0 += cpp) {
        const int ncols = min(cpp, a.D - col0);
        const int upr = ncols * esz / 16;              // 16-byte chunks of each row in this pass (at most 16)
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
            if (c * 32 >= ncols) break;                // the same for the whole warp (tcgen05.ld is warp-wide)
            uint32_t o[2][32];
            tmem_ld32(o_taddr + col0 + c * 32, o[0]);
            if ((c + 1) * 32 < ncols) tmem_ld32(o_taddr + col0 + (c + 1) * 32, o[1]);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                if ((c + k) * 32 >= ncols) break;
                uint32_t w[32];
                pack_out32(a.out_dt, o[k], inv, w);
                const int nb = min(32, ncols - (c + k) * 32) * esz;
                uint4* sd = reinterpret_cast<uint4*>(stage + lane * kStagePitch + (c + k) * 32 * esz);
#pragma unroll
                for (int v = 0; v < 8; ++v)
                    if (v * 16 < nb) sd[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
            }
        }
        __syncwarp();
        // two rows per store instruction: lanes 0-15 row r, lanes 16-31 row r + 1, lane & 15 the 16-byte chunk
        const int chunk = lane & 15;
#pragma unroll
        for (int r = 0; r < 32; r += 2) {
            const int rr = r + (lane >> 4);
            uint8_t* d = reinterpret_cast<uint8_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(dst), rr));
            if (d != nullptr && chunk < upr)
                *reinterpret_cast<uint4*>(d + col0 * esz + chunk * 16) =
                    *reinterpret_cast<const uint4*>(stage + rr * kStagePitch + chunk * 16);
        }
        __syncwarp();
    }
}

// max of 32 values with three-input max instructions (a tree: 16 instructions, depth 4)
__device__ __forceinline__ float max32(const uint32_t (&r)[32]) {
    float m[11];
#pragma unroll
    for (int i = 0; i < 10; ++i) m[i] = fmax3(__uint_as_float(r[3 * i]), __uint_as_float(r[3 * i + 1]), __uint_as_float(r[3 * i + 2]));
    m[10] = fmaxf(__uint_as_float(r[30]), __uint_as_float(r[31]));
    const float a0 = fmax3(m[0], m[1], m[2]), a1 = fmax3(m[3], m[4], m[5]), a2 = fmax3(m[6], m[7], m[8]);
    return fmax3(fmax3(a0, a1, a2), m[9], m[10]);
}

constexpr uint32_t kBias = 0x4B400000u;          // the bits of 1.5 * 2^23
constexpr float kBiasF = 12582912.0f;

// 16 consecutive 32-bit columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// ---- host side ---------------------------------------------------------------------------------------------------------

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// A 4-D map of 128-row boxes over B sequences of a tensor with D features per (token, head). Strides in bytes.
// order 0: dims (D, S, H, B) (packed [B, H, S, D]); order 1: dims (D, H, S, B) (token-major rows: the head stride is the
// smaller one). Returns an empty string, or why the map cannot be made (TMA wants a 16-byte aligned base and strides).
inline std::string make_rows_map(CUtensorMap* m, const void* base, bool int8, int64_t D, int64_t S, int64_t H, int64_t B,
                                 int64_t tok_bytes, int64_t head_bytes, int64_t seq_bytes, int order) {
    auto enc = tensor_map_encoder();
    if (!enc) return "cuTensorMapEncodeTiled is not available from the driver";
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (tok_bytes & 15) || (head_bytes & 15) || (seq_bytes & 15))
        return "not 16-byte aligned";
    const int es = int8 ? 1 : 2;
    cuuint64_t dims[4];
    cuuint64_t strides[3];
    cuuint32_t box[4];
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    dims[0] = (cuuint64_t) D;
    dims[3] = (cuuint64_t) B;
    strides[2] = (cuuint64_t) (B > 1 ? seq_bytes : (order == 0 ? head_bytes * H : tok_bytes * S));
    box[0] = (cuuint32_t) (128 / es);
    box[3] = 1;
    if (order == 0) {
        dims[1] = (cuuint64_t) S; dims[2] = (cuuint64_t) H;
        strides[0] = (cuuint64_t) tok_bytes; strides[1] = (cuuint64_t) head_bytes;
        box[1] = 128; box[2] = 1;
    } else {
        dims[1] = (cuuint64_t) H; dims[2] = (cuuint64_t) S;
        strides[0] = (cuuint64_t) head_bytes; strides[1] = (cuuint64_t) tok_bytes;
        box[1] = 1; box[2] = 128;
    }
    const CUresult r = enc(m, int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                           const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return "cuTensorMapEncodeTiled failed (" + std::to_string((int) r) + ")";
    return {};
}

}  // namespace h3
