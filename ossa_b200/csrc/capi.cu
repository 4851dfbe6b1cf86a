// C ABI entry points (declared in include/ossa_b200.h): argument validation,
// workspace carving and kernel dispatch.  Validation happens before any CUDA
// call, so a rejected request never touches the device.
#include "../../include/ossa_b200.h"
#include "kernels.h"

#include <atomic>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string>

namespace ossa {
namespace {
std::atomic<unsigned long long> g_launches{0};
}
void note_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }
}  // namespace ossa

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

}  // namespace

namespace ossa {
// Lets other translation units of the library report a message through
// ossa_last_error_string.
void set_error_message(const char* msg) { g_last_error = msg; }

int device_sm_count() {
    constexpr int kMaxDev = 64;
    static std::atomic<int> cached[kMaxDev];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 148;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}
}  // namespace ossa

namespace {

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return OSSA_OK;
    return fail(OSSA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr size_t kAlign = 256;
size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

bool valid_dtype(int d) { return d == OSSA_F32 || d == OSSA_BF16; }

int check_heads(int B, int H, int Hkv, int N) {
    if (B < 0 || H <= 0 || Hkv <= 0 || N < 0)
        return fail(OSSA_ERR_INVALID, "bad shape B=%d H=%d Hkv=%d N=%d", B, H, Hkv, N);
    if (H % Hkv != 0)
        return fail(OSSA_ERR_INVALID, "H=%d is not a multiple of Hkv=%d", H, Hkv);
    if ((long long)B * H > (1ll << 30) || N > (1 << 30))
        return fail(OSSA_ERR_UNSUPPORTED, "shape too large B=%d H=%d N=%d", B, H, N);
    return OSSA_OK;
}

// Workspace: [counters 256 B][q' fp32][k' fp32][tensor-core selection scratch]
// [split selection scratch (few query rows only)].  The counters block
// (fallback row count, status word) sits at offset 0 so ossa_router_status can
// find it for any shape.
struct RouterLayout {
    size_t qp_off, kp_off, tc_off, split_off, total;
};

// Fewer query rows than one tensor-core tile against more keys than one split
// range: the split selector (select_split.cu) instead of the CTA-per-128-rows
// one, which would give each row a single thread.
constexpr long long kSplitMaxRows = 128;
constexpr int kSplitMinKeys = 2048;
bool split_shape(int B, int H, int Nq, int Nk) {
    return (long long)B * H * Nq < kSplitMaxRows && Nk >= kSplitMinKeys;
}

constexpr size_t kCountersBytes = 256;

// Nq query rows per (b, h) against Nk keys per (b, kv head); K = 0 for scoring
// without selection.  own_kp = false: the caller holds the projected keys (the
// decode key cache), so the workspace has no k' region.
RouterLayout router_layout(int B, int H, int Hkv, int Nq, int Nk, int r, int K, bool own_kp = true) {
    RouterLayout l;
    const size_t qp = (size_t)B * H * Nq * r * sizeof(float);
    const size_t kp = own_kp ? (size_t)B * Hkv * Nk * r * sizeof(float) : 0;
    l.qp_off = kCountersBytes;
    l.kp_off = l.qp_off + align_up(qp);
    l.tc_off = l.kp_off + align_up(kp);
    l.split_off = l.tc_off + (r == 64 ? align_up(ossa::router_tc_workspace_bytes(B, H, Hkv, Nq, Nk, K)) : 0);
    l.total = l.split_off + (K > 0 && split_shape(B, H, Nq, Nk)
                                 ? align_up(ossa::split_select_workspace_bytes((long long)B * H * Nq, Nk, K))
                                 : 0);
    return l;
}

// The tensor-core selector serves r = 64, K <= 128 and at least one full tile of
// query and key rows; OSSA_ROUTER_SELECT=exact forces the CUDA-core exact selector
// of score_topk.cu in place of it and of the split selector (all produce identical
// indices; the switch exists to cross-check them).
bool use_tensor_core_select(int B, int H, int Hkv, int Nq, int Nk, int r, int K) {
    const char* env = getenv("OSSA_ROUTER_SELECT");
    if (env && env[0] == 'e') return false;
    return ossa::router_tc_supported(r, K) && (long long)B * Hkv * Nk >= 128 && (long long)B * H * Nq >= 128;
}

bool supported_r(int r) { return r == 16 || r == 32 || r == 64 || r == 128; }

// The oracle selection runs on the tensor-core kernel for head_dim 128, K <= 128
// and at least one full tile of query and key rows; OSSA_ORACLE_SELECT=exact
// forces the CUDA-core exact selector (identical indices; the switch exists to
// cross-check them).
bool use_tensor_core_oracle(int B, int H, int Hkv, int N, int D, int K) {
    const char* env = getenv("OSSA_ORACLE_SELECT");
    if (env && env[0] == 'e') return false;
    return ossa::oracle_tc_supported(D, K) && (long long)B * Hkv * N >= 128 && (long long)B * H * N >= 128;
}

size_t oracle_workspace_bytes(int B, int H, int Hkv, int N, int D, int K, int dtype) {
    if (!use_tensor_core_oracle(B, H, Hkv, N, D, K)) return kCountersBytes;
    return kCountersBytes + align_up(ossa::oracle_tc_workspace_bytes(B, H, Hkv, N, K, dtype));
}

int check_rows(int Nq, int Nk, int q0) {
    if (Nq < 0 || q0 < 0 || (long long)q0 + Nq > (1ll << 30))
        return fail(OSSA_ERR_INVALID, "bad query rows Nq=%d q_start=%d (keys %d)", Nq, q0, Nk);
    return OSSA_OK;
}

int check_router(const void* q, const void* k, int dtype, const float* wq, const float* wk,
                 const float* pos_bias, int B, int H, int Hkv, int Nq, int Nk, int q0, int D, int r,
                 int seq_len_cfg, int K, const void* out, void* ws, size_t ws_bytes, bool own_kp = true) {
    int st = check_heads(B, H, Hkv, Nk);
    if (st) return st;
    if ((st = check_rows(Nq, Nk, q0))) return st;
    if (!valid_dtype(dtype)) return fail(OSSA_ERR_INVALID, "bad dtype %d", dtype);
    if (D <= 0) return fail(OSSA_ERR_INVALID, "bad head_dim D=%d", D);
    if (!supported_r(r)) return fail(OSSA_ERR_UNSUPPORTED, "proj_dim r=%d not in {16,32,64,128}", r);
    if (seq_len_cfg <= 0 || seq_len_cfg > (1 << 28))
        return fail(OSSA_ERR_INVALID, "bad seq_len_cfg %d", seq_len_cfg);
    if ((long long)B * H * Nq == 0) return OSSA_OK;
    if (Nk == 0) return fail(OSSA_ERR_INVALID, "query rows need at least one key (Nk=0)");
    if (!q || !k || !wq || !wk || !pos_bias || !out)
        return fail(OSSA_ERR_INVALID, "null pointer argument");
    if (!aligned16(q) || !aligned16(k) || !aligned16(out))
        return fail(OSSA_ERR_INVALID, "q, k and the output must be 16-byte aligned");
    const RouterLayout l = router_layout(B, H, Hkv, Nq, Nk, r, K, own_kp);
    if (!ws || ws_bytes < l.total || !aligned16(ws))
        return fail(OSSA_ERR_WORKSPACE, "workspace of %zu bytes (16-byte aligned) required, got %zu",
                    l.total, ws ? ws_bytes : (size_t)0);
    return OSSA_OK;
}

// Whether the tensor-core selector takes this call with its query operand made
// straight from the bf16 q rows (router_qtc.cu) and canonical q' only for the rows
// that need it.  OSSA_QPROJ=canonical projects every row first (the same indices;
// the switch exists to cross-check the two).
bool lazy_qproj(const ossa::ProjectArgs& pa, int B, int H, int Hkv, int Nq, int Nk, int r, int K) {
    const char* env = getenv("OSSA_QPROJ");
    if (env && env[0] == 'c') return false;
    return use_tensor_core_select(B, H, Hkv, Nq, Nk, r, K) && ossa::qproj_tc_supported(pa);
}

int project_both(const void* q, const void* k, int dtype, const float* wq, const float* wk,
                 int B, int H, int Hkv, int Nq, int Nk, int D, int r, void* ws, cudaStream_t stream,
                 float** qp_out, float** kp_out) {
    const RouterLayout l = router_layout(B, H, Hkv, Nq, Nk, r, 0);  // qp_off, kp_off do not depend on K
    char* base = static_cast<char*>(ws);
    float* qp = reinterpret_cast<float*>(base + l.qp_off);
    float* kp = reinterpret_cast<float*>(base + l.kp_off);
    ossa::ProjectArgs pa{q, wq, qp, (long long)B * H * Nq, D, r, dtype};
    int st = cuda_status(ossa::launch_project(pa, stream), "q projection launch");
    if (st) return st;
    ossa::ProjectArgs pk{k, wk, kp, (long long)B * Hkv * Nk, D, r, dtype};
    st = cuda_status(ossa::launch_project(pk, stream), "k projection launch");
    if (st) return st;
    *qp_out = qp;
    *kp_out = kp;
    return OSSA_OK;
}

// Selection of Nq query rows from projected q' (B*H*Nq, r) and k' (B*Hkv*Nk, r):
// the tensor-core selector, the split selector (few rows, many keys) or the
// CTA selector; `l` is the workspace layout of the call.
// qproj: the q projection, not launched yet, when the caller leaves q' to the
// tensor-core selector (lazy_qproj); any other selector projects it first.
int select_rows(const float* qp, const float* kp, const float* pos_bias, int B, int H, int Hkv, int Nq, int Nk,
                int r, int seq_len_cfg, int K, int causal, int q_start, int32_t* idx_out, void* workspace,
                const RouterLayout& l, cudaStream_t s, const ossa::ProjectArgs* qproj = nullptr) {
    const float scale = (float)(1.0 / sqrt((double)r));
    if (use_tensor_core_select(B, H, Hkv, Nq, Nk, r, K)) {
        ossa::RouterTcArgs a{qp, kp, pos_bias, seq_len_cfg, B, H, Hkv, Nk, K, causal ? 1 : 0, scale,
                             idx_out, static_cast<char*>(workspace) + l.tc_off,
                             reinterpret_cast<int*>(workspace)};
        a.Nq = Nq;
        a.q0 = q_start;
        a.qproj = qproj;
        return cuda_status(ossa::launch_router_tc(a, s), "tensor-core router top-K launch");
    }
    if (qproj) {
        int st = cuda_status(ossa::launch_project(*qproj, s), "q projection launch");
        if (st) return st;
    }
    const char* env = getenv("OSSA_ROUTER_SELECT");
    if (split_shape(B, H, Nq, Nk) && !(env && env[0] == 'e')) {
        ossa::SplitSelectArgs a{qp, kp, pos_bias, seq_len_cfg, B, H, Hkv, Nk, r, K, scale, causal ? 1 : 0,
                                idx_out, Nq, q_start, static_cast<char*>(workspace) + l.split_off};
        return cuda_status(ossa::launch_split_select(a, s), "split router top-K launch");
    }
    ossa::ScoreTopkArgs a{qp, kp, ossa::kF32, pos_bias, seq_len_cfg, B, H, Hkv, Nk, r, K, scale,
                          causal ? 1 : 0, idx_out};
    a.Nq = Nq;
    a.q0 = q_start;
    return cuda_status(ossa::launch_score_topk(a, s), "router top-K launch");
}

}  // namespace

extern "C" {

const char* ossa_version(void) { return "0.1.0"; }

const char* ossa_last_error_string(void) { return g_last_error.c_str(); }

uint64_t ossa_launch_count(void) { return (uint64_t)ossa::g_launches.load(std::memory_order_relaxed); }

int ossa_topk_attention_fwd_rows(const void* q, const void* k, const void* v, const void* indices,
                                 int idx_is_64, int dtype, int B, int H, int Hkv, int Nq, int Nk, int D, int K,
                                 float scale, int causal, int q_start, void* out, ossa_stream_t stream) {
    int st = check_heads(B, H, Hkv, Nk);
    if (st) return st;
    if ((st = check_rows(Nq, Nk, q_start))) return st;
    if (!valid_dtype(dtype)) return fail(OSSA_ERR_INVALID, "bad dtype %d", dtype);
    if (D != 16 && D != 32 && D != 64 && D != 128 && D != 256)
        return fail(OSSA_ERR_UNSUPPORTED, "head_dim D=%d not in {16,32,64,128,256}", D);
    if (K < 0) return fail(OSSA_ERR_INVALID, "bad K=%d", K);
    if (idx_is_64 != 0 && idx_is_64 != 1) return fail(OSSA_ERR_INVALID, "idx_is_64 must be 0 or 1");
    if (!isfinite(scale)) return fail(OSSA_ERR_INVALID, "scale must be finite");
    if ((long long)B * H * Nq == 0) return OSSA_OK;
    if (Nk == 0) return fail(OSSA_ERR_INVALID, "query rows need at least one key (Nk=0)");
    if (!q || !k || !v || !out || (K > 0 && !indices))
        return fail(OSSA_ERR_INVALID, "null pointer argument");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return fail(OSSA_ERR_INVALID, "q, k, v and out must be 16-byte aligned");
    if (K > 0 && !aligned16(indices)) return fail(OSSA_ERR_INVALID, "indices must be 16-byte aligned");
    ossa::GatherArgs a{q, k, v, indices, out, idx_is_64, dtype, B, H, Hkv, Nk, D, K, scale, causal ? 1 : 0};
    a.Nq = Nq;
    a.q0 = q_start;
    return cuda_status(ossa::launch_gather_attn(a, static_cast<cudaStream_t>(stream)),
                       "topk attention launch");
}

int ossa_topk_attention_fwd(const void* q, const void* k, const void* v, const void* indices,
                            int idx_is_64, int dtype, int B, int H, int Hkv, int N, int D, int K,
                            float scale, int causal, void* out, ossa_stream_t stream) {
    return ossa_topk_attention_fwd_rows(q, k, v, indices, idx_is_64, dtype, B, H, Hkv, N, N, D, K, scale, causal,
                                        0, out, stream);
}

int ossa_router_status(const void* workspace, int* fallback_rows, int* status) {
    if (!workspace || !aligned16(workspace)) return fail(OSSA_ERR_INVALID, "bad workspace pointer");
    int h[2] = {0, 0};
    int st = cuda_status(cudaMemcpy(h, workspace, sizeof(h), cudaMemcpyDeviceToHost), "status read");
    if (st) return st;
    if (fallback_rows) *fallback_rows = h[0];
    if (status) *status = h[1];
    return OSSA_OK;
}

size_t ossa_router_workspace_size_rows(int B, int H, int Hkv, int Nq, int Nk, int r, int K) {
    if (B < 0 || H <= 0 || Hkv <= 0 || Nq < 0 || Nk < 0 || r <= 0) return 0;
    return router_layout(B, H, Hkv, Nq, Nk, r, K).total;
}

size_t ossa_router_workspace_size(int B, int H, int Hkv, int N, int r, int K) {
    return ossa_router_workspace_size_rows(B, H, Hkv, N, N, r, K);
}

int ossa_router_topk_rows(const void* q, const void* k, int dtype, const float* wq, const float* wk,
                          const float* pos_bias, int B, int H, int Hkv, int Nq, int Nk, int D, int r,
                          int seq_len_cfg, int K, int causal, int q_start, int32_t* idx_out, void* workspace,
                          size_t workspace_bytes, ossa_stream_t stream) {
    int st = check_router(q, k, dtype, wq, wk, pos_bias, B, H, Hkv, Nq, Nk, q_start, D, r, seq_len_cfg, K,
                          idx_out, workspace, workspace_bytes);
    if (st) return st;
    if (K <= 0) return fail(OSSA_ERR_INVALID, "bad K=%d", K);
    if (!ossa::score_topk_supported(r, K))
        return fail(OSSA_ERR_UNSUPPORTED, "top-K selection supports K <= 160 (got K=%d)", K);
    if ((long long)B * H * Nq == 0) return OSSA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    st = cuda_status(cudaMemsetAsync(workspace, 0, kCountersBytes, s), "workspace counters reset");
    if (st) return st;
    const RouterLayout l = router_layout(B, H, Hkv, Nq, Nk, r, K);
    float* qp = reinterpret_cast<float*>(static_cast<char*>(workspace) + l.qp_off);
    float* kp = reinterpret_cast<float*>(static_cast<char*>(workspace) + l.kp_off);
    const ossa::ProjectArgs pa{q, wq, qp, (long long)B * H * Nq, D, r, dtype};
    if (lazy_qproj(pa, B, H, Hkv, Nq, Nk, r, K)) {
        const ossa::ProjectArgs pk{k, wk, kp, (long long)B * Hkv * Nk, D, r, dtype};
        if ((st = cuda_status(ossa::launch_project(pk, s), "k projection launch"))) return st;
        return select_rows(qp, kp, pos_bias, B, H, Hkv, Nq, Nk, r, seq_len_cfg, K, causal, q_start, idx_out,
                           workspace, l, s, &pa);
    }
    st = project_both(q, k, dtype, wq, wk, B, H, Hkv, Nq, Nk, D, r, workspace, s, &qp, &kp);
    if (st) return st;
    return select_rows(qp, kp, pos_bias, B, H, Hkv, Nq, Nk, r, seq_len_cfg, K, causal, q_start, idx_out, workspace,
                       l, s);
}

size_t ossa_router_workspace_size_kp(int B, int H, int Hkv, int Nq, int Nk, int r, int K) {
    if (B < 0 || H <= 0 || Hkv <= 0 || Nq < 0 || Nk < 0 || r <= 0) return 0;
    return router_layout(B, H, Hkv, Nq, Nk, r, K, false).total;
}

int ossa_router_project_keys(const void* k, int dtype, const float* wk, long long rows, int D, int r,
                             float* kp_out, ossa_stream_t stream) {
    if (!valid_dtype(dtype)) return fail(OSSA_ERR_INVALID, "bad dtype %d", dtype);
    if (rows < 0 || D <= 0) return fail(OSSA_ERR_INVALID, "bad shape rows=%lld D=%d", rows, D);
    if (!supported_r(r)) return fail(OSSA_ERR_UNSUPPORTED, "proj_dim r=%d not in {16,32,64,128}", r);
    if (rows == 0) return OSSA_OK;
    if (!k || !wk || !kp_out) return fail(OSSA_ERR_INVALID, "null pointer argument");
    if (!aligned16(k) || !aligned16(kp_out)) return fail(OSSA_ERR_INVALID, "k and kp_out must be 16-byte aligned");
    ossa::ProjectArgs pk{k, wk, kp_out, rows, D, r, dtype};
    return cuda_status(ossa::launch_project(pk, static_cast<cudaStream_t>(stream)), "k projection launch");
}

int ossa_router_topk_rows_kp(const void* q, int dtype, const float* wq, const float* kp, const float* pos_bias,
                             int B, int H, int Hkv, int Nq, int Nk, int D, int r, int seq_len_cfg, int K,
                             int causal, int q_start, int32_t* idx_out, void* workspace, size_t workspace_bytes,
                             ossa_stream_t stream) {
    int st = check_router(q, kp, dtype, wq, wq, pos_bias, B, H, Hkv, Nq, Nk, q_start, D, r, seq_len_cfg, K,
                          idx_out, workspace, workspace_bytes, false);
    if (st) return st;
    if (K <= 0) return fail(OSSA_ERR_INVALID, "bad K=%d", K);
    if (!ossa::score_topk_supported(r, K))
        return fail(OSSA_ERR_UNSUPPORTED, "top-K selection supports K <= 160 (got K=%d)", K);
    if ((long long)B * H * Nq == 0) return OSSA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    st = cuda_status(cudaMemsetAsync(workspace, 0, kCountersBytes, s), "workspace counters reset");
    if (st) return st;
    const RouterLayout l = router_layout(B, H, Hkv, Nq, Nk, r, K, false);
    float* qp = reinterpret_cast<float*>(static_cast<char*>(workspace) + l.qp_off);
    const ossa::ProjectArgs pa{q, wq, qp, (long long)B * H * Nq, D, r, dtype};
    if (lazy_qproj(pa, B, H, Hkv, Nq, Nk, r, K))
        return select_rows(qp, kp, pos_bias, B, H, Hkv, Nq, Nk, r, seq_len_cfg, K, causal, q_start, idx_out,
                           workspace, l, s, &pa);
    st = cuda_status(ossa::launch_project(pa, s), "q projection launch");
    if (st) return st;
    return select_rows(qp, kp, pos_bias, B, H, Hkv, Nq, Nk, r, seq_len_cfg, K, causal, q_start, idx_out, workspace,
                       l, s);
}

int ossa_router_topk(const void* q, const void* k, int dtype, const float* wq, const float* wk,
                     const float* pos_bias, int B, int H, int Hkv, int N, int D, int r,
                     int seq_len_cfg, int K, int causal, int32_t* idx_out, void* workspace,
                     size_t workspace_bytes, ossa_stream_t stream) {
    return ossa_router_topk_rows(q, k, dtype, wq, wk, pos_bias, B, H, Hkv, N, N, D, r, seq_len_cfg, K, causal, 0,
                                 idx_out, workspace, workspace_bytes, stream);
}

int ossa_router_topk_sorted(const void* q, const void* k, int dtype, const float* wq, const float* wk,
                            const float* pos_bias, int B, int H, int Hkv, int N, int D, int r, int seq_len_cfg,
                            int K, int causal, int32_t* idx_out, void* workspace, size_t workspace_bytes,
                            ossa_stream_t stream) {
    int st = ossa_router_topk(q, k, dtype, wq, wk, pos_bias, B, H, Hkv, N, D, r, seq_len_cfg, K, causal, idx_out,
                              workspace, workspace_bytes, stream);
    if (st) return st;
    if ((long long)B * H * N == 0) return OSSA_OK;
    if (!ossa::sort_rows_supported(r, K))
        return fail(OSSA_ERR_UNSUPPORTED, "score-ordered rows support K <= 256 (got K=%d)", K);
    // the selection left the canonical k' in the workspace, and q' too unless the
    // tensor-core selector made only the rows it needed: then q' is projected here
    const RouterLayout l = router_layout(B, H, Hkv, N, N, r, K);
    char* base = static_cast<char*>(workspace);
    const ossa::ProjectArgs pa{q, wq, reinterpret_cast<float*>(base + l.qp_off), (long long)B * H * N, D, r, dtype};
    if (lazy_qproj(pa, B, H, Hkv, N, N, r, K) &&
        (st = cuda_status(ossa::launch_project(pa, static_cast<cudaStream_t>(stream)), "q projection launch")))
        return st;
    ossa::SortRowsArgs a{reinterpret_cast<const float*>(base + l.qp_off),
                         reinterpret_cast<const float*>(base + l.kp_off),
                         pos_bias, seq_len_cfg, H, Hkv, N, r, K, (float)(1.0 / sqrt((double)r)),
                         (long long)B * H * N, idx_out};
    return cuda_status(ossa::launch_sort_rows(a, static_cast<cudaStream_t>(stream)), "score-order launch");
}

int ossa_router_score(const void* q, const void* k, int dtype, const float* wq, const float* wk,
                      const float* pos_bias, int B, int H, int Hkv, int N, int D, int r,
                      int seq_len_cfg, float* scores_out, void* workspace, size_t workspace_bytes,
                      ossa_stream_t stream) {
    int st = check_router(q, k, dtype, wq, wk, pos_bias, B, H, Hkv, N, N, 0, D, r, seq_len_cfg, 0,
                          scores_out, workspace, workspace_bytes);
    if (st) return st;
    if ((long long)B * H * N == 0) return OSSA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float *qp = nullptr, *kp = nullptr;
    st = project_both(q, k, dtype, wq, wk, B, H, Hkv, N, N, D, r, workspace, s, &qp, &kp);
    if (st) return st;
    ossa::ScoreDenseArgs a{qp, kp, pos_bias, seq_len_cfg, B, H, Hkv, N, r,
                           (float)(1.0 / sqrt((double)r)), scores_out};
    return cuda_status(ossa::launch_score_dense(a, s), "router score launch");
}

int ossa_oracle_topk(const void* q, const void* k, int dtype, int B, int H, int Hkv, int N, int D,
                     float scale, int K, int causal, int32_t* idx_out, ossa_stream_t stream) {
    int st = check_heads(B, H, Hkv, N);
    if (st) return st;
    if (!valid_dtype(dtype)) return fail(OSSA_ERR_INVALID, "bad dtype %d", dtype);
    if (!supported_r(D))
        return fail(OSSA_ERR_UNSUPPORTED, "oracle selection supports head_dim in {16,32,64,128}, got %d", D);
    if (K <= 0) return fail(OSSA_ERR_INVALID, "bad K=%d", K);
    if (!ossa::score_topk_supported(D, K))
        return fail(OSSA_ERR_UNSUPPORTED, "top-K selection supports K <= 160 (got K=%d)", K);
    if (!isfinite(scale)) return fail(OSSA_ERR_INVALID, "scale must be finite");
    if ((long long)B * H * N == 0) return OSSA_OK;
    if (!q || !k || !idx_out) return fail(OSSA_ERR_INVALID, "null pointer argument");
    if (!aligned16(q) || !aligned16(k) || !aligned16(idx_out))
        return fail(OSSA_ERR_INVALID, "q, k and the output must be 16-byte aligned");
    ossa::ScoreTopkArgs a{q, k, dtype, nullptr, 1, B, H, Hkv, N, D, K, scale, causal ? 1 : 0, idx_out};
    return cuda_status(ossa::launch_score_topk(a, static_cast<cudaStream_t>(stream)),
                       "oracle top-K launch");
}

size_t ossa_router_distill_workspace_size(int B, int H, int Hkv, int N, int r) {
    if (B < 0 || H <= 0 || Hkv <= 0 || N < 0 || !supported_r(r)) return 0;
    const size_t rq = (size_t)B * H * N * r * sizeof(float), rk = (size_t)B * Hkv * N * r * sizeof(float);
    return kCountersBytes + 2 * align_up(rq) + 2 * align_up(rk) +
           align_up(ossa::distill_loss_parts(B, H, N) * sizeof(float));
}

int ossa_router_distill_grad(const void* q, const void* k, int dtype, const float* wq, const float* wk,
                             const float* pos_bias, int B, int H, int Hkv, int N, int D, int r, int seq_len_cfg,
                             const int32_t* targets, int K, float* loss_out, float* dwq, float* dwk,
                             float* dpos_bias, void* workspace, size_t workspace_bytes, ossa_stream_t stream) {
    int st = check_heads(B, H, Hkv, N);
    if (st) return st;
    if (!valid_dtype(dtype)) return fail(OSSA_ERR_INVALID, "bad dtype %d", dtype);
    if (D <= 0) return fail(OSSA_ERR_INVALID, "bad head_dim D=%d", D);
    if (!supported_r(r)) return fail(OSSA_ERR_UNSUPPORTED, "proj_dim r=%d not in {16,32,64,128}", r);
    if (seq_len_cfg <= 0 || seq_len_cfg > (1 << 28)) return fail(OSSA_ERR_INVALID, "bad seq_len_cfg %d", seq_len_cfg);
    if (K < 0) return fail(OSSA_ERR_INVALID, "bad K=%d", K);
    if ((long long)B * H * N == 0) return fail(OSSA_ERR_INVALID, "empty input (the mean loss is undefined)");
    if (!q || !k || !wq || !wk || !pos_bias || !loss_out || !dwq || !dwk || !dpos_bias || (K > 0 && !targets))
        return fail(OSSA_ERR_INVALID, "null pointer argument");
    if (!aligned16(q) || !aligned16(k)) return fail(OSSA_ERR_INVALID, "q and k must be 16-byte aligned");
    const size_t need = ossa_router_distill_workspace_size(B, H, Hkv, N, r);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
        return fail(OSSA_ERR_WORKSPACE, "workspace of %zu bytes (16-byte aligned) required, got %zu", need,
                    workspace ? workspace_bytes : (size_t)0);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* w = static_cast<char*>(workspace) + kCountersBytes;
    const size_t rq = (size_t)B * H * N * r * sizeof(float), rk = (size_t)B * Hkv * N * r * sizeof(float);
    float* qp = reinterpret_cast<float*>(w);
    float* kp = reinterpret_cast<float*>(w + align_up(rq));
    float* dqp = reinterpret_cast<float*>(w + align_up(rq) + align_up(rk));
    float* dkp = reinterpret_cast<float*>(w + 2 * align_up(rq) + align_up(rk));
    float* parts = reinterpret_cast<float*>(w + 2 * align_up(rq) + 2 * align_up(rk));
    ossa::ProjectArgs pa{q, wq, qp, (long long)B * H * N, D, r, dtype};
    if ((st = cuda_status(ossa::launch_project(pa, s), "q projection launch"))) return st;
    ossa::ProjectArgs pk{k, wk, kp, (long long)B * Hkv * N, D, r, dtype};
    if ((st = cuda_status(ossa::launch_project(pk, s), "k projection launch"))) return st;
    if ((st = cuda_status(cudaMemsetAsync(dwq, 0, (size_t)r * D * sizeof(float), s), "gradient reset"))) return st;
    if ((st = cuda_status(cudaMemsetAsync(dwk, 0, (size_t)r * D * sizeof(float), s), "gradient reset"))) return st;
    if ((st = cuda_status(cudaMemsetAsync(dpos_bias, 0, (size_t)2 * seq_len_cfg * sizeof(float), s),
                          "gradient reset")))
        return st;
    ossa::DistillArgs a{q, k, dtype, qp, kp, pos_bias, seq_len_cfg, B, H, Hkv, N, D, r, targets, K,
                        dqp, dkp, dpos_bias, dwq, dwk, parts, loss_out};
    return cuda_status(ossa::launch_distill(a, s), "router distillation launch");
}

int ossa_rope_to_heads(const void* x, const void* cos, const void* sin, int cs_batched, int dtype, int B, int N,
                       int Hx, int D, void* out, ossa_stream_t stream) {
    if (!valid_dtype(dtype)) return fail(OSSA_ERR_INVALID, "bad dtype %d", dtype);
    if (B < 0 || N < 0 || Hx <= 0 || D <= 0 || D % 8 != 0)
        return fail(OSSA_ERR_INVALID, "bad shape B=%d N=%d heads=%d D=%d (D must be a multiple of 8)", B, N, Hx, D);
    if ((long long)B * N == 0) return OSSA_OK;
    if (!x || !out || (!cos) != (!sin)) return fail(OSSA_ERR_INVALID, "null pointer argument");
    if (!aligned16(x) || !aligned16(out) || (cos && (!aligned16(cos) || !aligned16(sin))))
        return fail(OSSA_ERR_INVALID, "x, cos, sin and out must be 16-byte aligned");
    ossa::RopeArgs a{x, cos, sin, cs_batched ? 1 : 0, dtype, B, N, Hx, D, out};
    return cuda_status(ossa::launch_rope_heads(a, static_cast<cudaStream_t>(stream)), "rope launch");
}

size_t ossa_oracle_workspace_size(int B, int H, int Hkv, int N, int D, int K, int dtype) {
    if (B < 0 || H <= 0 || Hkv <= 0 || N < 0 || D <= 0 || K <= 0 || !valid_dtype(dtype)) return 0;
    return oracle_workspace_bytes(B, H, Hkv, N, D, K, dtype);
}

int ossa_oracle_topk_ws(const void* q, const void* k, int dtype, int B, int H, int Hkv, int N, int D,
                        float scale, int K, int causal, int32_t* idx_out, void* workspace,
                        size_t workspace_bytes, ossa_stream_t stream) {
    int st = check_heads(B, H, Hkv, N);
    if (st) return st;
    if (!valid_dtype(dtype)) return fail(OSSA_ERR_INVALID, "bad dtype %d", dtype);
    if (!supported_r(D))
        return fail(OSSA_ERR_UNSUPPORTED, "oracle selection supports head_dim in {16,32,64,128}, got %d", D);
    if (K <= 0) return fail(OSSA_ERR_INVALID, "bad K=%d", K);
    if (!ossa::score_topk_supported(D, K))
        return fail(OSSA_ERR_UNSUPPORTED, "top-K selection supports K <= 160 (got K=%d)", K);
    if (!isfinite(scale)) return fail(OSSA_ERR_INVALID, "scale must be finite");
    if ((long long)B * H * N == 0) return OSSA_OK;
    if (!q || !k || !idx_out) return fail(OSSA_ERR_INVALID, "null pointer argument");
    if (!aligned16(q) || !aligned16(k) || !aligned16(idx_out))
        return fail(OSSA_ERR_INVALID, "q, k and the output must be 16-byte aligned");
    const size_t need = oracle_workspace_bytes(B, H, Hkv, N, D, K, dtype);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
        return fail(OSSA_ERR_WORKSPACE, "workspace of %zu bytes (16-byte aligned) required, got %zu", need,
                    workspace ? workspace_bytes : (size_t)0);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    st = cuda_status(cudaMemsetAsync(workspace, 0, kCountersBytes, s), "workspace counters reset");
    if (st) return st;
    if (!use_tensor_core_oracle(B, H, Hkv, N, D, K)) {
        ossa::ScoreTopkArgs a{q, k, dtype, nullptr, 1, B, H, Hkv, N, D, K, scale, causal ? 1 : 0, idx_out};
        return cuda_status(ossa::launch_score_topk(a, s), "oracle top-K launch");
    }
    ossa::OracleTcArgs a{q, k, dtype, B, H, Hkv, N, K, causal ? 1 : 0, scale, idx_out,
                         static_cast<char*>(workspace) + kCountersBytes, reinterpret_cast<int*>(workspace)};
    return cuda_status(ossa::launch_oracle_tc(a, s), "tensor-core oracle top-K launch");
}

}  // extern "C"
