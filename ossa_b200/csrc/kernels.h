// Internal launcher interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ossa {

enum DType { kF32 = 0, kBF16 = 1 };

// Counts successful kernel launches (ossa_launch_count); every launcher calls it.
void note_launch(int n = 1);

// Sets the message ossa_last_error_string returns on this thread.
void set_error_message(const char* msg);

// Streaming multiprocessors of the current device (queried once per device).
int device_sm_count();

// Tensor map of a (rows x cols) row-major matrix of 16-bit values (bf16, else fp16)
// in box_rows x 64-column boxes with the 128-byte swizzle (a row of cols > 64 takes
// cols / 64 boxes).
bool make_row_map_16(CUtensorMap* map, const void* base, bool bf16, unsigned long long rows, int cols,
                     int box_rows);

struct GatherArgs {
    const void* q;
    const void* k;
    const void* v;
    const void* idx;
    void* out;
    int idx_is_64;
    int dtype;
    int B, H, Hkv, N, D, K;
    float scale;
    int causal;
    int Nq = 0;  // query rows per (b, h); 0 means N (queries are the keys' positions)
    int q0 = 0;  // position of query row 0 in the key sequence
};
cudaError_t launch_gather_attn(const GatherArgs& a, cudaStream_t stream);

// out[row][c] = fmaf-chain over d = 0..D-1 of x[row][d] * w[c][d], for c < R.
struct ProjectArgs {
    const void* x;   // (rows, D), dtype
    const float* w;  // (R, D) fp32
    float* out;      // (rows, R) fp32
    long long rows;
    int D, R, dtype;
};
cudaError_t launch_project(const ProjectArgs& a, cudaStream_t stream);

// The tensor-core selector's query operand straight from bf16 q rows (D = 128,
// r = 64; router_qtc.cu): q16 (fp16, scaled per row), rowinfo (multiplier, error
// bound covering the canonical q') and rowub, from the per-(b, kv head) key
// statistics.  The canonical q' itself is not written.
struct QPrepArgs {
    const void* x;   // bf16 q rows [rows][128]
    const float* w;  // Wq [64][128]
    float* wt;       // written: Wq transposed, [128][64] (read by the selector's on-demand q' rows)
    long long rows;
    void* q16;
    float2* rowinfo;
    float* rowub;
    const uint32_t* stats;
    const uint32_t* gstats;
    int* status;  // bit 32: a bounded wait of the kernel expired
    int H, Hkv, Nq;
    float scale;
};
bool qproj_tc_supported(const ProjectArgs& a);
cudaError_t launch_qproj_tc(const QPrepArgs& a, cudaStream_t stream);

// Exact fp32 causal/full top-K over score(i,j) = dot(qrows_i, krows_j) * scale
// (+ pos_bias[clamp(i - j + L, 0, 2L - 1)] when bias != nullptr).
// qrows: (B*H*N, R), krows: (B*Hkv*N, R), both `dtype`.
struct ScoreTopkArgs {
    const void* qrows;
    const void* krows;
    int dtype;
    const float* bias;
    int L;
    int B, H, Hkv, N, R, K;
    float scale;
    int causal;
    int32_t* out;  // (B*H*Nq, K)
    int Nq = 0;    // query rows per (b, h); 0 means N (queries are the keys' positions)
    int q0 = 0;    // position of query row 0 in the key sequence
};
cudaError_t launch_score_topk(const ScoreTopkArgs& a, cudaStream_t stream);
bool score_topk_supported(int R, int K);

// The same exact selection for a few query rows against many keys (decode):
// one warp per (row, range of keys), then one warp per row over the ranges'
// winners.  qrows (B*H*Nq, R), krows (B*Hkv*N, R) fp32; ws holds
// split_select_workspace_bytes(B*H*Nq, N, K).
struct SplitSelectArgs {
    const float* qrows;
    const float* krows;
    const float* bias;  // nullptr: no position term
    int L;
    int B, H, Hkv, N, R, K;
    float scale;
    int causal;
    int32_t* out;  // (B*H*Nq, K)
    int Nq;        // query rows per (b, h)
    int q0;        // position of query row 0 in the key sequence
    void* ws;
};
// RoPE (x*cos + rotate_half(x)*sin, rounded as the eager ops) fused with the
// (B, N, Hx, D) -> (B, Hx, N, D) layout change; cosv == nullptr: layout only.
struct RopeArgs {
    const void* x;     // (B, N, Hx, D)
    const void* cosv;  // (1 or B, N, D) or nullptr
    const void* sinv;
    int cs_batched;    // cos/sin carry a batch dimension
    int dtype;
    int B, N, Hx, D;
    void* out;         // (B, Hx, N, D)
};
cudaError_t launch_rope_heads(const RopeArgs& a, cudaStream_t stream);

bool split_select_supported(int R, int K);
size_t split_select_workspace_bytes(long long rows, int N, int K);
cudaError_t launch_split_select(const SplitSelectArgs& a, cudaStream_t stream);

// Reorders each selected index row (ascending keys, -1 padded) in place to
// (canonical score desc, key asc), -1 padding last: torch.topk's order.
// qp (rows, R), kp (B*Hkv*N, R) fp32 projections; rows = B*H*N.
struct SortRowsArgs {
    const float* qp;
    const float* kp;
    const float* bias;  // nullptr: no position term
    int L;
    int H, Hkv, N, R, K;
    float scale;
    long long rows;
    int32_t* idx;       // (rows, K)
};
bool sort_rows_supported(int R, int K);
cudaError_t launch_sort_rows(const SortRowsArgs& a, cudaStream_t stream);

// Router distillation loss (BCE over all (i, j) against 0/1 targets) and the
// gradients of q', k', pos_bias and the projection weights, streamed in tiles.
struct DistillArgs {
    const void* q;        // (B*H*N, D) dtype: the rows q' was projected from
    const void* k;        // (B*Hkv*N, D) dtype
    int dtype;
    const float* qp;      // (B*H*N, R) canonical q'
    const float* kp;      // (B*Hkv*N, R) canonical k'
    const float* bias;    // (2L,)
    int L;
    int B, H, Hkv, N, D, R;
    const int32_t* tgt;   // (B*H*N, K) target key lists (-1 padded)
    int K;
    float* dqp;           // (B*H*N, R) out
    float* dkp;           // (B*Hkv*N, R) out
    float* dbias;         // (2L,) accumulated (zero it first)
    float* dwq;           // (R, D) accumulated (zero it first)
    float* dwk;           // (R, D) accumulated (zero it first)
    float* loss_part;     // distill_loss_parts(B, H, N) per-CTA loss sums
    float* loss_out;      // (1,) mean loss
};
size_t distill_loss_parts(int B, int H, int N);
cudaError_t launch_distill(const DistillArgs& a, cudaStream_t stream);

// Dense fp32 scores (B, H, N, N) with the same score definition, no mask.
struct ScoreDenseArgs {
    const float* qrows;
    const float* krows;
    const float* bias;
    int L;
    int B, H, Hkv, N, R;
    float scale;
    float* out;
};
cudaError_t launch_score_dense(const ScoreDenseArgs& a, cudaStream_t stream);

}  // namespace ossa

namespace ossa {

// Tensor-core (tcgen05) router selection, r = 64, K <= 128.  qp32/kp32: canonical fp32
// projections; ws: router_tc_workspace_bytes of scratch; counters: two ints
// (rows sent to the exact fallback, status word: 0 = ok, nonzero = a bounded
// wait expired), zeroed by the caller before the launch.
struct RouterTcArgs {
    const float* qp32;
    const float* kp32;
    const float* bias;
    int L;
    int B, H, Hkv, N, K, causal;
    float scale;
    int32_t* out;
    void* ws;
    int* counters;
    int Nq = 0;  // query rows per (b, h); 0 means N (queries are the keys' positions)
    int q0 = 0;  // position of query row 0 in the key sequence
    // When set (qproj_tc_supported), q' is not projected up front: the selector's
    // query operand comes from launch_qproj_tc and the canonical q' rows are computed
    // into qp32 (qproj->out) only for the rows that need them.
    const ProjectArgs* qproj = nullptr;
};
bool router_tc_supported(int r, int K);
size_t router_tc_workspace_bytes(int B, int H, int Hkv, int Nq, int N, int K);
cudaError_t launch_router_tc(const RouterTcArgs& a, cudaStream_t stream);

// The oracle selector (exact scaled q.k scores, no pos_bias) on the same
// tensor-core kernel, for head_dim kOracleD: fp16 scores find the candidates,
// fp32 canonical scores decide them (indices identical to launch_score_topk).
constexpr int kOracleD = 128;
struct OracleTcArgs {
    const void* q;  // [B, H, N, D] rows, dtype
    const void* k;  // [B, Hkv, N, D] rows, dtype
    int dtype;
    int B, H, Hkv, N, K, causal;
    float scale;
    int32_t* out;
    void* ws;       // oracle_tc_workspace_bytes
    int* counters;  // two ints, zeroed before the launch
};
bool oracle_tc_supported(int D, int K);
size_t oracle_tc_workspace_bytes(int B, int H, int Hkv, int N, int K, int dtype);
cudaError_t launch_oracle_tc(const OracleTcArgs& a, cudaStream_t stream);

}  // namespace ossa
