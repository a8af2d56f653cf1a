/* h3sage.h - the C ABI of libh3sage.so: SageAttention v1 on NVIDIA B200 (sm_100a), as a run-time-loaded plugin.
 *
 * A drop-in for the reference's kernels/sage.cpp (maxfridbe/sycl_minimax_h3): libh3cuda.so (like libh3sycl.so,
 * kernels/h3sycl.cpp:1683-1701) dlopens it from its own directory and resolves h3sage_attention and h3sage_error.
 * The SYCL queue pointer of the reference becomes a pointer to a cudaStream_t; the work is queued on that stream and
 * not waited for.
 *
 * What it computes, per head h and query row i (non-causal):
 *   out[h, i, :] = sum_j softmax_j( (q[h,i,:] . k[h,j,:]) * qscale[h, i/block] * kscale[h, j/block] * scale ) v[h, j, :]
 * q, k int8 [H, S, D] (k already has its channel mean taken out; that changes no softmax), v and out half [H, S, D],
 * scales float32 [H, ceil(S/block)]. The int8 dot products run on tcgen05 kind::i8 with int32 sums in tensor memory,
 * P.V on kind::f16 with fp32 sums.
 */
#ifndef H3SAGE_H
#define H3SAGE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The reason of the last failure of this library (kernels/sage.cpp:28). Process-wide, like the reference's. */
const char* h3sage_error(void);

/* 0 on success, else -1 with the reason in h3sage_error(). D must be 64 or 128 (kernels/sage.cpp:33); block a
 * multiple of 64 (kernels/sage.cpp:34); S * H * D < 2^31 (kernels/sage.cpp:35).
 * (kernels/sage.cpp:31-32) */
int h3sage_attention(void* stream, const int8_t* q, const int8_t* k, const void* v, void* out, const float* qscale,
                     const float* kscale, int block, int64_t S, int64_t H, int64_t D, float scale);

/* ---- additions without a counterpart in the reference ----------------------------------------------------------- */

/* The same attention with v read in place and the output written in place, which is how libh3cuda.so calls it (no
 * relayout copies): v element (s, h, d) at v + s*v_tok + h*v_head + d (half), out element (s, h, d) at
 * out + s*out_tok + h*out_head + d in out_dt (0 float32, 1 half, 2 bfloat16; values rounded through half first).
 * err: a device int the kernel ORs a nonzero code into when one of its waits gives up after wait_ns nanoseconds
 * (NULL: the plugin's own word, read by h3sage_check). */
int h3sage_attention_strided(void* stream, const int8_t* q, const int8_t* k, const void* v, int64_t v_tok,
                             int64_t v_head, void* out, int out_dt, int64_t out_tok, int64_t out_head,
                             const float* qscale, const float* kscale, int block, int64_t S, int64_t H, int64_t D,
                             float scale, int* err, uint64_t wait_ns);

/* h3sage_attention_strided with the output rows spread over the P ranks of a Ulysses group (P <= 8, S a multiple of
 * P): the row of token s goes to out_peers[s / (S/P)] (that rank's token shard, in this or another GPU's memory,
 * already offset to this rank's head columns) at row s % (S/P), each stored as the attention produces it. */
int h3sage_attention_peers(void* stream, const int8_t* q, const int8_t* k, const void* v, int64_t v_tok, int64_t v_head,
                           void* const* out_peers, int P, int out_dt, int64_t out_tok, int64_t out_head,
                           const float* qscale, const float* kscale, int block, int64_t S, int64_t H, int64_t D,
                           float scale, int* err, uint64_t wait_ns);

/* Waits for the stream and reports, as -1 with h3sage_error(), a kernel wait of this plugin that gave up since the
 * last check (the reference reports such failures only through its queue's wait). */
int h3sage_check(void* stream);

#ifdef __cplusplus
}
#endif
#endif
