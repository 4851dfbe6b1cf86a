/*
 * ossa_oracle.c — CPU oracle for the routed sparse-attention selection path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load this library, and only as the checker.  The product
 * path (ossa_b200/) never calls it.
 *
 * It restates, in plain C, the selection the reference performs with PyTorch:
 *   ContentRouter.score        ossa/router.py:171-190
 *     q' = q Wq^T, k' = k Wk^T (nn.Linear, no bias)            router.py:179-180
 *     logits = (q' k'^T) * (1/sqrt(r))                           router.py:181-182
 *     + pos_bias[clamp(i - j + seq_len, 0, 2*seq_len - 1)]       router.py:184-189
 *   causal mask + torch.topk   ossa/bench/sparse_forward.py:180, 200-202
 *   oracle selector q k^T/sqrt(D)  ossa/bench/sparse_forward.py:194-196
 * with every floating-point step pinned so that a GPU kernel can match it bit for
 * bit (the reference's BLAS summation order is unspecified):
 *   projection  p[c]  = fmaf-chain over d = 0..D-1 of x[d] * W[c][d], from 0.0f
 *   dot(i,j)          = fmaf-chain over c = 0..R-1 of a_i[c] * b_j[c], from 0.0f
 *   score(i,j)        = fl(fl(dot * scale) + bias[...])   (two roundings, as
 *                       torch's `* scale` then `+ bias` round)
 * and the selection rule made total: the K largest scores by (value desc, key
 * index asc), NaN ranked above +inf as torch.topk ranks it, emitted in
 * ascending key order, padded with -1 when fewer than K keys are eligible.
 *
 * Build: oracle/build.py (gcc -O2 -ffp-contract=off -fopenmp -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef __FAST_MATH__
#error "the oracle must not be compiled with -ffast-math (it would license re-association)"
#endif

static uint32_t order_key(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    if (f != f) b = 0x7fc00000u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

/* out[row][c] = fmaf chain over d of x[row][d] * w[c][d]. */
void orc_project(const float* x, const float* w, int64_t rows, int D, int R, float* out) {
    int64_t row;
#pragma omp parallel for schedule(static)
    for (row = 0; row < rows; ++row) {
        const float* xr = x + row * (int64_t)D;
        for (int c = 0; c < R; ++c) {
            const float* wr = w + (int64_t)c * D;
            float acc = 0.0f;
            for (int d = 0; d < D; ++d) acc = fmaf(xr[d], wr[d], acc);
            out[row * R + c] = acc;
        }
    }
}

static float score_one(const float* a, const float* b, int R, float scale, const float* bias,
                       int L, int i, int j) {
    float acc = 0.0f;
    for (int c = 0; c < R; ++c) acc = fmaf(a[c], b[c], acc);
    volatile float s = acc * scale; /* rounded product, never contracted */
    float r = s;
    if (bias) {
        int bi = i - j + L;
        if (bi < 0) bi = 0;
        if (bi > 2 * L - 1) bi = 2 * L - 1;
        r = r + bias[bi];
    }
    return r;
}

/* Dense scores, (B, H, N, N), no mask: the materialised ContentRouter.score. */
void orc_scores(const float* arows, const float* brows, const float* bias, int L, int B, int H,
                int Hkv, int N, int R, float scale, float* out) {
    const int G = H / Hkv;
    int64_t t, total = (int64_t)B * H * N;
#pragma omp parallel for schedule(static)
    for (t = 0; t < total; ++t) {
        const int64_t bh = t / N;
        const int i = (int)(t % N);
        const int b = (int)(bh / H), h = (int)(bh % H), g = h / G;
        const float* a = arows + t * R;
        const float* kb = brows + ((int64_t)b * Hkv + g) * N * R;
        float* o = out + t * (int64_t)N;
        for (int j = 0; j < N; ++j) o[j] = score_one(a, kb + (int64_t)j * R, R, scale, bias, L, i, j);
    }
}

static int cmp_i32_asc(const void* x, const void* y) {
    int32_t a = *(const int32_t*)x, b = *(const int32_t*)y;
    return a < b ? -1 : (a > b ? 1 : 0);
}

/* Partially orders keys[0..n) so that its K largest occupy keys[0..K). */
static void select_top(uint64_t* keys, int n, int K) {
    int lo = 0, hi = n - 1;
    int target = K - 1;
    while (lo < hi) {
        uint64_t pivot = keys[lo + (hi - lo) / 2];
        int l = lo, r = hi;
        while (l <= r) {
            while (keys[l] > pivot) ++l;
            while (keys[r] < pivot) --r;
            if (l <= r) {
                uint64_t tmp = keys[l];
                keys[l] = keys[r];
                keys[r] = tmp;
                ++l;
                --r;
            }
        }
        if (target <= r) hi = r;
        else if (target >= l) lo = l;
        else break;
    }
}

/* Selects row t = (b*H + h)*N + i, whose a-vector is `a`, into out[0..K)
 * (and scores_out when not NULL). */
static void topk_row(const float* a, const float* brows, const float* bias, int L, int H, int Hkv,
                     int N, int R, float scale, int K, int causal, int64_t t, uint64_t* keys,
                     int32_t* sel, int32_t* out, float* scores_out) {
    const int G = H / Hkv;
    const int64_t bh = t / N;
    const int i = (int)(t % N);
    const int b = (int)(bh / H), h = (int)(bh % H), g = h / G;
    const float* kb = brows + ((int64_t)b * Hkv + g) * N * R;
    const int n = causal ? i + 1 : N;
    for (int j = 0; j < n; ++j) {
        const float s = score_one(a, kb + (int64_t)j * R, R, scale, bias, L, i, j);
        keys[j] = ((uint64_t)order_key(s) << 32) | (uint64_t)(0xffffffffu - (uint32_t)j);
    }
    const int m = n < K ? n : K;
    if (m > 0 && m < n) select_top(keys, n, m);
    for (int p = 0; p < m; ++p) sel[p] = (int32_t)(0xffffffffu - (uint32_t)(keys[p] & 0xffffffffu));
    qsort(sel, (size_t)m, sizeof(int32_t), cmp_i32_asc);
    for (int p = 0; p < K; ++p) out[p] = p < m ? sel[p] : -1;
    if (scores_out) {
        for (int p = 0; p < K; ++p)
            scores_out[p] = p < m ? score_one(a, kb + (int64_t)sel[p] * R, R, scale, bias, L, i, sel[p]) : NAN;
    }
}

/*
 * Top-K selection for every row (b, h, i).
 *   arows: (B*H*N, R)   brows: (B*Hkv*N, R)   bias: NULL or (2L)
 *   out:   (B*H*N, K) int32, ascending key order, -1 padding.
 * If scores_out is not NULL it also receives the selected keys' fp32 scores in
 * the same slots (NaN in padded slots).
 */
void orc_topk(const float* arows, const float* brows, const float* bias, int L, int B, int H,
              int Hkv, int N, int R, float scale, int K, int causal, int32_t* out,
              float* scores_out) {
    int64_t t, total = (int64_t)B * H * N;
#pragma omp parallel
    {
        uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(N > 0 ? N : 1));
        int32_t* sel = (int32_t*)malloc(sizeof(int32_t) * (size_t)(K > 0 ? K : 1));
#pragma omp for schedule(dynamic, 16)
        for (t = 0; t < total; ++t)
            topk_row(arows + t * R, brows, bias, L, H, Hkv, N, R, scale, K, causal, t, keys, sel,
                     out + t * (int64_t)K, scores_out ? scores_out + t * (int64_t)K : NULL);
        free(keys);
        free(sel);
    }
}

/*
 * The same selection for a list of rows only: rows[r] = (b*H + h)*N + i.
 * arows holds the a-vectors of the listed rows only, (nrows, R); out is (nrows, K).
 */
void orc_topk_rows(const float* arows, const float* brows, const float* bias, int L, int B, int H,
                   int Hkv, int N, int R, float scale, int K, int causal, const int64_t* rows,
                   int64_t nrows, int32_t* out) {
    (void)B;
    int64_t r;
#pragma omp parallel
    {
        uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(N > 0 ? N : 1));
        int32_t* sel = (int32_t*)malloc(sizeof(int32_t) * (size_t)(K > 0 ? K : 1));
#pragma omp for schedule(dynamic, 1)
        for (r = 0; r < nrows; ++r) {
            topk_row(arows + r * R, brows, bias, L, H, Hkv, N, R, scale, K, causal, rows[r], keys, sel,
                     out + r * (int64_t)K, NULL);
        }
        free(keys);
        free(sel);
    }
}
