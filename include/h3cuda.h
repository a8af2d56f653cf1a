/* h3cuda.h - the C ABI of libh3cuda.so: the denoiser self-attention path of MiniMax H3 on NVIDIA B200 (sm_100a).
 *
 * A drop-in for the attention subset of the reference's kernels/h3sycl.h (maxfridbe/sycl_minimax_h3): the same names,
 * signatures, element-type codes and error conventions, with SYCL queues replaced by CUDA streams and USM by cudaMalloc.
 * Each declaration cites the reference declaration it replaces (file:line inside the reference project).
 *
 * Every data pointer is a device pointer of the context's GPU. Kernels are asynchronous: a call returns once its work
 * is queued on the context's stream, and the stream is in order, so a later call sees an earlier call's result;
 * h3s_read and h3s_wait are the points that wait. Functions returning int give 0, or -1 with the reason in
 * h3s_last_error() (per thread). Functions returning a pointer give NULL on failure, same.
 *
 * Environment (read when a context is made; same meanings as the reference's, kernels/h3sycl.cpp:216-235):
 *   H3S_ATTN=onednn (or =sdpa)  never use the int8 Sage path
 *   H3S_SAGE_MIN_S             sequences at least this long use Sage (default 8192)
 *   H3S_MEM_FRACTION           allocation cap as a fraction of the card (default 0.94)
 *   H3S_PROFILE                wait after every attention phase and report its time on stderr
 *   H3S_POISON                 fill new buffers with 0xff bytes (NaN) to expose reads of unwritten memory
 *   H3S_WAIT_MS                limit of every wait inside a kernel (default 2000); past it the kernel stops and
 *                              h3s_wait reports the failure
 */
#ifndef H3CUDA_H
#define H3CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types of floating-point tensors (kernels/h3sycl.h:21) */
enum { H3S_F32 = 0, H3S_F16 = 1, H3S_BF16 = 2 };

/* kernels/h3sycl.h:23 */
const char* h3s_last_error(void);

/* ---- context ---------------------------------------------------------------------------------------------------- */

/* A context on the first GPU with its own stream (kernels/h3sycl.h:28). */
void* h3s_open(void);
/* The GPUs CUDA sees; name, memory size and PCI address "0000:0b:00.0" of one (kernels/h3sycl.h:31-32). */
int h3s_gpu_count(void);
int h3s_gpu_info(int index, char* name, int name_len, uint64_t* mem_bytes, char* pci, int pci_len);
/* A context on GPU `index` with its own stream (kernels/h3sycl.h:33). */
void* h3s_open_gpu(int index);
/* A context around an existing stream: `stream` points to a cudaStream_t (PyTorch: the handle of
 * torch.cuda.current_stream()), which is copied; the current device is the context's GPU (kernels/h3sycl.h:36). */
void* h3s_create(void* stream);
/* Waits for the stream, frees the scratch buffers and everything still allocated with h3s_alloc (kernels/h3sycl.h:38). */
void h3s_destroy(void* ctx);
/* kernels/h3sycl.h:40 */
const char* h3s_device_name(void* ctx);

/* ---- device memory (kernels/h3sycl.h:47-53) --------------------------------------------------------------------- */

/* Allocations are counted, and one that would pass the cap (0.94 of the card; H3S_MEM_FRACTION overrides) is refused
 * with an error. The attention's own scratch buffers count against the same cap. */
void* h3s_alloc(void* ctx, uint64_t bytes);
void h3s_free(void* ctx, void* p); /* waits for the stream first */
uint64_t h3s_mem_used(void* ctx);
uint64_t h3s_mem_cap(void* ctx);
/* What the whole card has free right now, every process counted. */
uint64_t h3s_mem_free(void* ctx);

/* ---- copies (kernels/h3sycl.h:56-61) ---------------------------------------------------------------------------- */

/* Host <-> device; both wait for the copy (and for the work queued before it). Thread-safe. */
int h3s_write(void* ctx, void* dst, const void* src_host, uint64_t bytes);
int h3s_read(void* ctx, void* dst_host, const void* src, uint64_t bytes);
/* Device to device, queued like a kernel. */
int h3s_copy(void* ctx, void* dst, const void* src, uint64_t bytes);
/* Waits until everything queued has run; reports an asynchronous error (a CUDA error, or a kernel wait that gave up). */
int h3s_wait(void* ctx);

/* ---- pinned host memory and uploads beside the kernels (kernels/h3sycl.h:65-71) --------------------------------- */

void* h3s_alloc_host(void* ctx, uint64_t bytes);
void h3s_free_host(void* ctx, void* p); /* waits for the uploads first */
/* Pinned host -> device on the context's copy stream; the kernels do not wait for it: call h3s_upload_wait before
 * using dst. src must come from h3s_alloc_host, dst must be device memory; anything else is refused. */
int h3s_upload(void* ctx, void* dst, const void* src_pinned, uint64_t bytes);
int h3s_upload_wait(void* ctx);

/* ---- attention (kernels/h3sycl.h:185-197) ----------------------------------------------------------------------- */

/* out = softmax(q . k^T / sqrt(D)) . v, per head. q, k, v: S token rows of H heads x D features, row s at element
 * s * stride (stride >= H * D; 3 * H * D when they sit inside the qkv linear's output), in type dt; out [S, H * D] in
 * out_dt, rounded through half. S >= H3S_SAGE_MIN_S (8192): SageAttention v1 (int8 q, k with per-64-row scales after
 * k's channel mean is taken out; libh3sage.so beside this library) for D = 64 or 128, as the reference's plugin
 * (kernels/sage.cpp:33); every other call, and every D from 1 to 128, fp16 SDPA. D > 128 returns -1: a narrowing of
 * the reference, whose fused path takes any D (kernels/h3sycl.cpp:1464-1573); the engine's heads are 128 (denoiser)
 * and 64 (VAE). S, H or D <= 0: nothing to do, returns 0. No score table is ever written: memory stays O(S * H * D).
 * (kernels/h3sycl.h:190-191) */
int h3s_attention(void* ctx, const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D,
                  int64_t stride, void* out, int out_dt);
/* B independent sequences of S tokens in one call: sequence b's rows start at row b * S of q, k, v and of out
 * [B * S, H * D]. Below the Sage threshold all sequences go in one launch; Sage takes them one at a time.
 * (kernels/h3sycl.h:196-197) */
int h3s_attention_batch(void* ctx, const void* q, const void* k, const void* v, int dt, int64_t B, int64_t S, int64_t H,
                        int64_t D, int64_t stride, void* out, int out_dt);

/* ---- the step before the attention (kernels/h3sycl.h:165-174) --------------------------------------------------- */

/* Per-head RMS norm, then the rotary position rotation, in place: what the denoiser runs on q and k right before
 * h3s_attention (engine/h3-core/src/dit.rs:347-348). x holds M token rows of H heads x D features, row m at element
 * m * stride (stride >= H * D), in type x_dt. Each head's features are normalised, s = sum of x*x in feature order,
 * inv = rsqrt(s / D + eps) (rounded once), x*inv*weight[i] (weight float [D]); then the pairs (i, rot_dim/2 + i),
 * i < rot_dim/2, are rotated by the token's angle, a' = a*cos - b*sin, b' = b*cos + a*sin, with (cos, sin) from cs
 * float [M, rot_dim/2, 2]. Features from rot_dim on are only normalised. rot_dim must be even, at most D, and leave an
 * even remainder, else -1. M, H or D <= 0: nothing to do, returns 0. Queued on the context's stream; no scratch. */
int h3s_rms_rope(void* ctx, void* x, int x_dt, int64_t M, int64_t H, int64_t D, int64_t stride, const float* weight,
                 float eps, const float* cs, int rot_dim);

/* ---- the block's linear layers (kernels/h3sycl.h:74-85) ----------------------------------------------------------- */

/* A linear layer with int8 weights and activations quantised on the fly (the int8_convrot checkpoints' layers: qkv,
 * out_proj, fc1, fc2 of every denoiser block, engine/h3-core/src/ops.rs:25-80):
 *
 *   x_rot = x . H           per group of `group` features, H the normalised Hadamard matrix h4 (x) h4 (x) ...
 *   s_r   = max(max|x_rot[r]| / 127, 1e-30)                  per row
 *   q     = clamp(rint(x_rot / s_r), -128, 127)              int8
 *   acc   = q . W^T                                          int32, on the tensor cores
 *   out   = acc * (s_r * wscale) + bias    (n_wscale = 1)    or   (acc * s_r) * wscale[n] + bias   (n_wscale = N)
 *
 * x [M, K] in x_dt; w int8 [N, K]; wscale float32 [n_wscale]; bias float32 [N] or NULL; out [M, N] in out_dt.
 * group = 0: no rotation; else a power of 2 up to 256 dividing K (as the reference accepts; 4^n is what checkpoints
 * use), else -1 "unsupported ConvRot group size". n_wscale must be 1 or N. M, K or N <= 0: nothing to do, returns 0.
 * Queued on the context's stream; the int8 copy of x is context scratch (grow-only, at most 1 GiB: longer inputs
 * run in row chunks). */
int h3s_int8_linear(void* ctx, const void* x, int x_dt, int64_t M, int64_t K, const int8_t* w, int64_t N,
                    const float* wscale, int64_t n_wscale, const float* bias, void* out, int out_dt, int group);

/* ---- the text encoder's attention (kernels/h3sycl.h:105-108) ---------------------------------------------------- */

/* Causal attention with grouped heads, for short sequences (the text encoder, engine/h3-core/src/te.rs:340-346): Hq
 * query heads share Hkv key/value heads (query head h reads key/value head h / (Hq / Hkv)). q rows of stride qs, k and
 * v rows of stride kvs (elements), type dt; out [L, Hq * D] in dt. Query i attends to keys 0..i with scores
 * q.k / sqrt(D), and every weight stays fp32 (nothing is rounded to half between the loads and the store).
 * D <= 256 and Hq a multiple of Hkv, else -1; L <= 0: nothing to do, returns 0. Queued on the context's stream. */
int h3s_attention_causal(void* ctx, const void* q, const void* k, const void* v, int dt, int64_t L, int64_t Hq,
                         int64_t Hkv, int64_t D, int64_t qs, int64_t kvs, void* out);

/* ---- additions without a counterpart in the reference ----------------------------------------------------------- */

/* The Ulysses exchange over peer memory, for one process per GPU on one node (NVLink/NVSwitch): a sequence of S
 * tokens sharded by tokens over P ranks (s = S/P rows each) is re-sharded by heads (h = H/P each) for the attention
 * and back, each rank storing straight into the other ranks' buffers.
 * h3s_ipc_handle: the 64-byte CUDA IPC handle of a buffer from h3s_alloc (its base pointer). h3s_ipc_open: another
 * process's buffer from its handle (NULL on failure); h3s_ipc_close undoes it. */
int h3s_ipc_handle(void* ctx, const void* ptr, void* handle);
void* h3s_ipc_open(void* ctx, const void* handle);
int h3s_ipc_close(void* ctx, void* ptr);
/* Forward: this rank's token rows of a qkv buffer, shard [s, 3*H*D] (q | k | v, es-byte elements: 2 or 4), into every
 * rank p's head-sharded buffer dst[p] = [P*s, 3*h*D]: heads p*h .. p*h+h-1 of each part, at rows rank*s .. rank*s+s-1.
 * Inverse: this rank's output out_heads [P*s, h*D] into every rank p's token rows dst[p] = [s, H*D] at columns
 * rank*h*D ... dst[rank] is this rank's own buffer, the others opened with h3s_ipc_open; P <= 8, H a multiple of P.
 * Queued on the context's stream; the ranks must meet (a collective on the same streams) before they overwrite what
 * another rank still reads and before they read what they received. */
int h3s_ulysses_push_qkv(void* ctx, const void* shard, int64_t s, int64_t H, int64_t D, int es, int P, int rank,
                         void* const* dst);
int h3s_ulysses_push_out(void* ctx, const void* out_heads, int64_t s, int64_t H, int64_t D, int es, int P, int rank,
                         void* const* dst);
/* h3s_attention of this rank's H heads over all S tokens (q, k, v as for h3s_attention) with the inverse exchange in
 * its epilogue: the output row of token t is stored straight into rank t / (S/P)'s token shard out_shards[t / (S/P)]
 * [S/P, P*H*D] (out_dt; this rank's own buffer or one opened with h3s_ipc_open) at row t % (S/P), columns
 * rank*H*D .. rank*H*D + H*D - 1. No separate output pass; the ranks must meet before another rank reads its shard. */
int h3s_attention_ulysses(void* ctx, const void* q, const void* k, const void* v, int dt, int64_t S, int64_t H,
                          int64_t D, int64_t stride, void* const* out_shards, int P, int rank, int out_dt);

/* The Sage pre-pass alone (kernels/h3sycl.cpp:1733-1761 as a callable step, for parity checks and for callers that
 * keep int8 q/k): iq, ik int8 [H, S, D]; sc float [2*H*nb + H*D] = q scales [H, nb], k scales [H, nb], k's channel
 * mean [H*D], nb = ceil(S / 64). D = 64 or 128. Queued on the context's stream. */
int h3s_sage_prepass(void* ctx, const void* q, const void* k, int dt, int64_t S, int64_t H, int64_t D, int64_t stride,
                     int8_t* iq, int8_t* ik, float* sc);
/* h3s_rms_rope(q, wq), h3s_rms_rope(k, wk), then h3s_sage_prepass, in one call with the same results bit for bit (q
 * and k are left normalised and rotated in place, as the two calls leave them). eps, cs and rot_dim as h3s_rms_rope,
 * with its refusals; D = 64 or 128, as h3s_sage_prepass. */
int h3s_sage_prepass_rope(void* ctx, void* q, void* k, int dt, int64_t S, int64_t H, int64_t D, int64_t stride,
                          const float* wq, const float* wk, float eps, const float* cs, int rot_dim, int8_t* iq,
                          int8_t* ik, float* sc);
/* A denoiser block's three calls before its output projection (engine/h3-core/src/dit.rs:347-350), in one:
 * h3s_rms_rope(q, wq), h3s_rms_rope(k, wk), h3s_attention(q, k, v, ..., out). The Sage path runs the fused pre-pass
 * above; the fp16 SDPA path normalises q and k first. q and k are left normalised and rotated in place either way;
 * the output is h3s_attention's on those rows. The refusals of both calls. */
int h3s_attention_rms_rope(void* ctx, void* q, void* k, const void* v, int dt, int64_t S, int64_t H, int64_t D,
                           int64_t stride, void* out, int out_dt, const float* wq, const float* wk, float eps,
                           const float* cs, int rot_dim);
/* The CUDA stream a context queues on (a cudaStream_t), for callers that order their own work with it. */
void* h3s_stream(void* ctx);
/* Self-test of the kernels' bounded waits: queues a kernel that waits `wait_ns` nanoseconds for an mbarrier nothing
 * arrives at, gives up, and records the failure like any kernel of this library; the following h3s_wait returns -1.
 * It faults nothing and leaves the context usable. */
int h3s_selftest_wait_timeout(void* ctx, uint64_t wait_ns);

/* The int8 Sage attention with no device allocation at all. No counterpart in the reference. For callers that cannot
 * allocate device memory when they call: code on a path that must not synchronise the device (cudaMalloc and cudaFree
 * may), and hosts whose device memory is wholly owned and budgeted by another allocator (a fixed cap, a caching
 * allocator), where a library allocating behind their back breaks the budget.
 * It computes what h3s_attention computes on its Sage path (K channel mean, int8 q/k per 64-row block, the tcgen05
 * kernel) for fp16 q, k, v rows at `stride` (16-byte aligned starts, stride a multiple of 8), D = 128, into out
 * [S, H*D] in out_dt, queued on *stream (stream points to a cudaStream_t; NULL: the legacy default stream). Its scratch
 * is a fixed array of 8 MiB + 128 KiB inside this library, which every GPU that loads the library holds until the
 * process exits: S*H*D <= 4,194,304 and H*D <= 16,384, else -1 with the limit in h3s_last_error(). The first call on
 * a device looks the array's address up (cudaGetSymbolAddress); make that first call before any stream capture.
 * err: a device int of the caller; each call first sets it to 0 on the stream, and a kernel whose wait gives up ORs a
 * nonzero code into it. Each GPU has its own copy of the array, shared by every call on that GPU: two calls on one GPU
 * whose work overlaps (different streams, not ordered by events) race on it, so order them. */
int h3s_attention_sage_static(void* stream, const void* q, const void* k, const void* v, int64_t S, int64_t H, int64_t D,
                              int64_t stride, void* out, int out_dt, int* err);

#ifdef __cplusplus
}
#endif
#endif
