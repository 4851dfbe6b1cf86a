/*
 * ossa_b200.h — C ABI of the Blackwell (sm_100a) routed sparse-attention hot path.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA stream
 * (passed as an opaque pointer, binary-compatible with cudaStream_t / CUstream).
 * Nothing here allocates device memory: the caller owns every buffer, including
 * outputs and the workspace whose size ossa_router_workspace_size() reports.
 * Work is enqueued on `stream` and returns without a host synchronisation.
 *
 * Tensors are contiguous row-major:
 *   q          (B, H,   N, D)
 *   k, v       (B, Hkv, N, D)   Hkv divides H; query head h reads kv head h / (H / Hkv),
 *                               the mapping repeat_interleave gives in
 *                               ossa/bench/sparse_forward.py:175-178. Hkv == H is the
 *                               already-repeated layout the reference passes around.
 *   indices    (B, H,   N, K)   int32 or int64
 *   out        (B, H,   N, D)   same dtype as q
 *
 * Status: every function returns OSSA_OK (0) or an error code; the message of the
 * last error on the calling thread is available from ossa_last_error_string().
 * No entry point calls exit/abort or traps on the device.
 */
#ifndef OSSA_B200_H
#define OSSA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define OSSA_API __attribute__((visibility("default")))
#else
#define OSSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* ossa_stream_t; /* a cudaStream_t; NULL is the legacy default stream */

enum ossa_status {
    OSSA_OK = 0,
    OSSA_ERR_INVALID = 1,     /* bad shape, dtype, pointer or alignment */
    OSSA_ERR_CUDA = 2,        /* a CUDA launch or runtime call failed */
    OSSA_ERR_WORKSPACE = 3,   /* workspace missing or smaller than required */
    OSSA_ERR_UNSUPPORTED = 4  /* valid request outside what the kernels implement */
};

enum ossa_dtype {
    OSSA_F32 = 0,
    OSSA_BF16 = 1
};

/* Library version string, e.g. "0.1.0". */
OSSA_API const char* ossa_version(void);

/* Message of the last failed call on this thread ("" if none). */
OSSA_API const char* ossa_last_error_string(void);

/*
 * Number of kernels this library has launched in the process so far (all
 * threads).  Diagnostic only, no counterpart in the reference: lets a caller
 * count the device launches a region of its own code issued.
 */
OSSA_API uint64_t ossa_launch_count(void);

/*
 * Gathered top-K attention forward, O(N*K*D).
 * Replaces topk_attention (ossa/triton_kernel.py:41-70) and the kernel it
 * launches (ossa/triton_kernel.py:80-167, 170-218); computes the same result as
 * sparse_attention_forward_chunked (ossa/sparse_attention.py:87-137):
 *   s_j   = (q_i . k_{idx_j}) * scale, masked to -inf when idx_j is outside [0, N)
 *           or (causal) idx_j > i;
 *   out_i = softmax(s) . V[idx], and 0 for a row whose every entry is masked.
 * dtype: OSSA_F32 or OSSA_BF16 for q, k, v and out (fp32 accumulation).
 * idx_is_64: 0 for int32 indices, 1 for int64.  D in {16, 32, 64, 128, 256}.
 */
OSSA_API int ossa_topk_attention_fwd(const void* q, const void* k, const void* v,
                            const void* indices, int idx_is_64, int dtype,
                            int B, int H, int Hkv, int N, int D, int K,
                            float scale, int causal, void* out,
                            ossa_stream_t stream);

/*
 * Bytes of workspace ossa_router_topk / ossa_router_score need for this shape.
 * Replaces nothing in the reference (its router materialises (B,H,N,N) logits,
 * ossa/router.py:182-189); the workspace holds the projected q'/k' rows and the
 * selector's scratch (fp16 copies, per-row bounds, position-bias windows; for
 * 64 < K <= 128 also the candidate lists, 2.5 KB per query row).  It depends on
 * K: size it with the K of the call.
 */
OSSA_API size_t ossa_router_workspace_size(int B, int H, int Hkv, int N, int r, int K);

/*
 * ContentRouter causal (or full) top-K key selection.
 * Replaces ContentRouter.score + masked_fill + torch.topk as the patched forward
 * runs them (ossa/router.py:171-190, ossa/bench/sparse_forward.py:185-202) and
 * ContentRouter.topk (ossa/router.py:202-203) when causal == 0.
 *   q', k'      = q Wq^T, k Wk^T  (wq, wk: (r, D) fp32, the nn.Linear weights)
 *   score(i,j)  = (q'_i . k'_j) * (1/sqrt(r)) + pos_bias[clamp(i - j + seq_len_cfg, 0, 2*seq_len_cfg - 1)]
 * Selection is in fp32: the K best keys by (score desc, key index asc) among
 * j <= i (causal) or all j.  Output row i lists the chosen key indices in
 * ascending order, padded with -1 when fewer than K keys are eligible.
 * q, k dtype: OSSA_F32 or OSSA_BF16 (converted exactly to fp32).
 */
OSSA_API int ossa_router_topk(const void* q, const void* k, int dtype,
                     const float* wq, const float* wk, const float* pos_bias,
                     int B, int H, int Hkv, int N, int D, int r, int seq_len_cfg,
                     int K, int causal, int32_t* idx_out,
                     void* workspace, size_t workspace_bytes,
                     ossa_stream_t stream);

/*
 * ossa_router_topk with each row in the order torch.topk returns.
 * Replaces ContentRouter.topk (ossa/router.py:202-203), whose result is
 * torch.topk(score, k).indices: keys by descending score.  Same arguments,
 * workspace and selected sets as ossa_router_topk; row i lists its keys by
 * (fp32 score desc, key index asc), -1 padding last.
 */
OSSA_API int ossa_router_topk_sorted(const void* q, const void* k, int dtype,
                                     const float* wq, const float* wk, const float* pos_bias,
                                     int B, int H, int Hkv, int N, int D, int r, int seq_len_cfg,
                                     int K, int causal, int32_t* idx_out,
                                     void* workspace, size_t workspace_bytes,
                                     ossa_stream_t stream);

/*
 * Diagnostic, no counterpart in the reference: reads (synchronously) the
 * counters block of a router workspace after ossa_router_topk has run on it:
 * the number of rows the tensor-core selector handed to its exact fallback
 * (near-ties or non-finite inputs) and the status word (0 = ok; nonzero = a
 * bounded device-side wait expired and the output is not valid).
 */
OSSA_API int ossa_router_status(const void* workspace, int* fallback_rows, int* status);

/*
 * Materialised router logits, (B, H, N, N) fp32, no causal mask.
 * Replaces ContentRouter.score / ContentRouter.forward (ossa/router.py:171-200)
 * with the same fp32 score definition ossa_router_topk selects on.
 */
OSSA_API int ossa_router_score(const void* q, const void* k, int dtype,
                      const float* wq, const float* wk, const float* pos_bias,
                      int B, int H, int Hkv, int N, int D, int r, int seq_len_cfg,
                      float* scores_out, void* workspace, size_t workspace_bytes,
                      ossa_stream_t stream);

/*
 * Oracle (exact dot-product) top-K selection, no router.
 * Replaces the oracle selector of the patched forward
 * (ossa/bench/sparse_forward.py:194-202): score(i,j) = (q_i . k_j) * scale in fp32,
 * then the same causal top-K rule and output layout as ossa_router_topk.
 */
OSSA_API int ossa_oracle_topk(const void* q, const void* k, int dtype,
                     int B, int H, int Hkv, int N, int D, float scale,
                     int K, int causal, int32_t* idx_out,
                     ossa_stream_t stream);

/*
 * The same oracle selection with a caller-provided workspace, which lets it run
 * on the tensor-core selector (head_dim 128, K <= 128): fp16 tensor-core scores
 * with a per-row error bound choose the candidates and the fp32 scores above
 * decide among them, so the indices equal ossa_oracle_topk's bit for bit.
 * Other shapes run the exact CUDA-core selector.  Replaces the same oracle
 * selector (ossa/bench/sparse_forward.py:194-202).  The workspace size depends on
 * the shape, K and dtype (ossa_oracle_workspace_size; 0 = invalid arguments);
 * its first 8 bytes are the counters ossa_router_status reads.
 */
OSSA_API size_t ossa_oracle_workspace_size(int B, int H, int Hkv, int N, int D, int K, int dtype);
OSSA_API int ossa_oracle_topk_ws(const void* q, const void* k, int dtype,
                                 int B, int H, int Hkv, int N, int D, float scale,
                                 int K, int causal, int32_t* idx_out,
                                 void* workspace, size_t workspace_bytes,
                                 ossa_stream_t stream);

/*
 * ossa_router_topk without a caller-provided workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory where
 * they launch this work (a host framework that owns every byte of device
 * memory and forbids allocation while enqueueing, or an FFI caller without a
 * device allocator).  It allocates nothing: the workspace is a fixed 32 MiB
 * array inside the library, held on every GPU that loads the library until the
 * process exits.  Shapes whose ossa_router_workspace_size exceeds 32 MiB are
 * rejected with OSSA_ERR_WORKSPACE.  The first call on each device looks up the
 * array's device address (make it before any stream capture); later calls look
 * it up again unless their stream is capturing.  `stream` must belong to the
 * current device.  All calls share the array: calls whose work overlaps on the
 * GPU race and must be serialised by the caller.  Same arguments and results as
 * ossa_router_topk otherwise.
 */
OSSA_API int ossa_router_topk_noalloc(const void* q, const void* k, int dtype,
                                      const float* wq, const float* wk, const float* pos_bias,
                                      int B, int H, int Hkv, int N, int D, int r, int seq_len_cfg,
                                      int K, int causal, int32_t* idx_out,
                                      ossa_stream_t stream);

/*
 * ossa_router_status for ossa_router_topk_noalloc, whose callers never see its
 * workspace: reads (synchronously) the counters of the last call on the current
 * device from the library's scratch array: rows handed to the exact fallback and
 * the status word (0 = ok; nonzero = a bounded device-side wait expired and that
 * call's indices are not valid).  No counterpart in the reference.
 */
OSSA_API int ossa_router_status_noalloc(int* fallback_rows, int* status);

/*
 * Query-row ranges for sequence sharding.  No counterpart in the reference,
 * which runs one process over the whole sequence
 * (ossa/bench/sparse_forward.py:157-229); these serve a rank that holds a
 * contiguous block of Nq query rows at positions q_start .. q_start+Nq-1
 * against all Nk keys of the sequence (k, v gathered from every rank):
 *   q, indices, out  (B, H, Nq, ...)      k, v  (B, Hkv, Nk, D)
 * Row l is query position q_start + l in the causal mask (j <= q_start + l)
 * and in the position bias (offset q_start + l - j).  With Nq == Nk and
 * q_start == 0 they are ossa_topk_attention_fwd, ossa_router_workspace_size and
 * ossa_router_topk exactly (those three call them).
 */
OSSA_API int ossa_topk_attention_fwd_rows(const void* q, const void* k, const void* v,
                                          const void* indices, int idx_is_64, int dtype,
                                          int B, int H, int Hkv, int Nq, int Nk, int D, int K,
                                          float scale, int causal, int q_start, void* out,
                                          ossa_stream_t stream);
OSSA_API size_t ossa_router_workspace_size_rows(int B, int H, int Hkv, int Nq, int Nk, int r, int K);
OSSA_API int ossa_router_topk_rows(const void* q, const void* k, int dtype,
                                   const float* wq, const float* wk, const float* pos_bias,
                                   int B, int H, int Hkv, int Nq, int Nk, int D, int r, int seq_len_cfg,
                                   int K, int causal, int q_start, int32_t* idx_out,
                                   void* workspace, size_t workspace_bytes,
                                   ossa_stream_t stream);

/*
 * Decode key cache.  No counterpart in the reference (its forward is
 * prefill-only, ossa/bench/sparse_forward.py:157-160).  A decoder projects each
 * new key once, k' = k Wk^T (ossa/router.py:180, the same fp32 chain as
 * ossa_router_topk), into a cache it owns, and selects against the cached rows:
 *   ossa_router_project_keys:  k (rows, D) dtype -> kp_out (rows, r) fp32
 *   ossa_router_topk_rows_kp:  ossa_router_topk_rows with the keys given as
 *       kp (B, Hkv, Nk, r) fp32 instead of k and wk; identical indices
 *   ossa_router_workspace_size_kp: its workspace (no k' region).
 */
OSSA_API size_t ossa_router_workspace_size_kp(int B, int H, int Hkv, int Nq, int Nk, int r, int K);
OSSA_API int ossa_router_project_keys(const void* k, int dtype, const float* wk, long long rows, int D, int r,
                                      float* kp_out, ossa_stream_t stream);
OSSA_API int ossa_router_topk_rows_kp(const void* q, int dtype, const float* wq, const float* kp,
                                      const float* pos_bias, int B, int H, int Hkv, int Nq, int Nk, int D, int r,
                                      int seq_len_cfg, int K, int causal, int q_start, int32_t* idx_out,
                                      void* workspace, size_t workspace_bytes, ossa_stream_t stream);

/*
 * Router distillation step without the (B, H, N, N) logits.
 * Replaces distillation_loss(router.score(q, k), dense, k=K) and its backward
 * (ossa/router.py:80-99 with router.py:171-190, as ossa/bench/content_train.py:141-148
 * trains the router): the mean over every (i, j) of BCE-with-logits between the
 * router score (the fp32 score ossa_router_topk selects on) and a 0/1 target that
 * marks the keys listed in row i of `targets` ((B, H, N, K) int32, -1 padded, any
 * order; the reference marks the top-K keys of the dense attention).  Writes the
 * loss (device float) and the gradients of wq, wk ((r, D) fp32) and pos_bias
 * ((2*seq_len_cfg,) fp32); q and k are inputs, not differentiated (the reference
 * detaches them).  Memory is linear in N: scores are recomputed tile by tile.
 */
OSSA_API size_t ossa_router_distill_workspace_size(int B, int H, int Hkv, int N, int r);
OSSA_API int ossa_router_distill_grad(const void* q, const void* k, int dtype,
                                      const float* wq, const float* wk, const float* pos_bias,
                                      int B, int H, int Hkv, int N, int D, int r, int seq_len_cfg,
                                      const int32_t* targets, int K, float* loss_out,
                                      float* dwq, float* dwk, float* dpos_bias,
                                      void* workspace, size_t workspace_bytes, ossa_stream_t stream);

/*
 * Rotary position embedding fused with the head transpose of the patched
 * layer (ossa/bench/sparse_forward.py:166-178: the q/k/v projections viewed as
 * (B, Hx, N, D), then Qwen2's apply_rotary_pos_emb on q and k).  Additive, for
 * the fused pre-processing of the patched layer:
 *   x   (B, N, Hx, D)  the linear projection's output rows
 *   cos, sin (1 or B, N, D) (cs_batched = 1 when they carry the batch), or both NULL
 *   out (B, Hx, N, D) = x*cos + rotate_half(x)*sin, rotate_half = cat(-x2, x1),
 *       each product and the sum rounded to the dtype as the eager ops round
 *       them (bit-identical to the PyTorch expression); without cos/sin a
 *       plain layout copy.
 * dtype OSSA_F32 or OSSA_BF16; D a multiple of 8; pointers 16-byte aligned.
 */
OSSA_API int ossa_rope_to_heads(const void* x, const void* cos, const void* sin, int cs_batched, int dtype,
                                int B, int N, int Hx, int D, void* out, ossa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* OSSA_B200_H */
