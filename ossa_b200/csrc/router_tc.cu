// Router top-K selection on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces ContentRouter.score + causal mask + torch.topk (ossa/router.py:171-190,
// ossa/bench/sparse_forward.py:180-202) for proj_dim r = 64 and K <= 128, with
// the same result as the exact CUDA-core selector: the K best keys by canonical
// fp32 score (fmaf chains, see score_topk.cu), lowest key index first on ties,
// emitted in ascending key order and -1 padded.
//
// Pipeline (one CTA = 128 query rows of one (b, h), one CTA per SM):
//  1. prep kernels turn the canonical fp32 projections q', k' into fp16 copies
//     scaled by powers of two (q' per row, k' per (b, kv head)) so every value
//     sits in [2^12, 2^13) at most (for bf16 q at head_dim 128 the query side
//     comes from the tensor-core operand kernel of router_qtc.cu instead, with
//     bounds that cover the canonical q', and the canonical q' rows are computed
//     in this file only for the rows that rescore or fall back), plus per row the
//     epilogue multiplier
//     m_i = scale * 2^-(e_q + e_k) and an error bound delta_i with
//     |approx score - canonical score| <= delta_i, built from the measured fp16
//     conversion errors dq_i = fp16(q'_i) - q'_i and dk_j (Cauchy-Schwarz):
//        delta_i = scale * (|q'_i| max|dk| + |dq_i| max|k'| + |dq_i| max|dk|)
//                  + scale * 2^-13 * |q'_i| * max_j |k'_j|   (fp32 accumulation: tensor core, fmaf chain)
//                  + 2^-22 * (max|bias| + scale * |q'_i| * max_j |k'_j|)   (final roundings)
//     and the call's pos_bias window images (window_table_kernel).
//  2. warp 0 (one thread) streams 128-key tiles of k'16 with TMA (128-byte
//     swizzle) through a 4- or 6-stage ring; warp 1 (one thread) issues
//     tcgen05.mma.kind::f16 128x128x64 into one of 4 TMEM accumulators; warp 2
//     (one thread) brings the tile's pos_bias window into the matching window
//     buffer with one bulk copy, completing on the same barrier as the MMA (each
//     of these threads spends tens of cycles per issued TMA/MMA instruction, so
//     the three streams are kept apart); eight epilogue warps (two per TMEM
//     lane quadrant, each owning 64 of the 128 columns; one query row per
//     thread) drain a finished accumulator with tcgen05.ld, release it, and score
//        s = acc * m_i + pos_bias[clamp(i - j + L, 0, 2L - 1)]
//     (the window holds the tile's 255 bias terms as four shifted copies with
//     the causal -inf already applied, so each thread reads the terms of 4
//     consecutive columns with one aligned 16-byte load).
//  3. Two passes over the same key tiles (the MMA runs twice; the epilogue is
//     the bottleneck, not the tensor core).  Pass 1 keeps, per row, the maximum
//     score of each column class: key index mod 128 (K <= 64), or key tile
//     parity x column, 256 classes (K <= 128).  The K-th largest class maximum
//     is a valid lower bound on the row's K-th best score (K distinct keys reach
//     it), so theta = bound - 2*delta_i can only drop keys outside the exact top
//     K.  Pass 2 appends every score >= theta to the thread's candidate sub-list
//     in global memory (about 1.3-1.4 K entries per row on random data).
//  4. final_select_kernel, one warp per row: the K-th best approximate score x_K
//     splits the candidates; entries above the split + 2*delta_i are certainly
//     selected, entries below x_K - 2*delta_i certainly not, and the few in
//     between are rescored with the canonical fp32 formula; the remaining slots
//     go to them by (score desc, j asc).  Output in ascending key order.
//     However wide the band (large |q'||k'| make delta wide), it is decided by
//     canonical rescoring of the row's candidates, never by a full-row scan.
//  5. Rows whose sub-list would overflow (massive near-ties) or whose inputs are
//     not finite are appended to a list and recomputed afterwards by an exact
//     warp-per-row selector (exact_rows_kernel).
//
// Every wait on an mbarrier is bounded (~1 s); on expiry the kernel records a
// nonzero status word, lets the other roles finish their bounded waits, waits
// for its own TMA loads and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cfloat>
#include <climits>
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "router_prep.cuh"
#include "select_warp.cuh"
#include "sm100.cuh"

namespace ossa {

namespace {

using namespace sm100;

constexpr int kR = 64;              // projection dim = MMA K
constexpr int kTileM = 128;         // query rows per CTA
constexpr int kTileN = 128;         // keys per MMA tile
constexpr int kAccBufs = 4;         // TMEM accumulators (128 columns each)
constexpr int kEpiWarps = 8;        // two per TMEM lane quadrant, 64 columns each
constexpr int kCtlWarps = 3;        // k' loads, MMA issue, window loads
constexpr int kThreads = 32 * (kCtlWarps + kEpiWarps);
constexpr int kHalfCols = kTileN / 2;
// pos_bias window of one tile, shared by the CTA: u[z] = bias term of column
// col for row `row` at z = col - row + 127, as four copies shifted by s = 0..3
// (copy s holds u[s .. s + kWinLen - 1]) so that every thread reads the terms of
// 4 consecutive columns with one aligned 16-byte load.
constexpr int kWinLen = 2 * kTileN - 4;  // 252 terms per copy (z <= 254)
constexpr int kWinCopy = kWinLen + 12;   // copy stride in floats, = 8 (mod 32): copies 8 banks apart
constexpr int kWinBytes = 4 * kWinCopy * 4;
static_assert(kWinCopy % 32 == 8 && (kWinLen * 4) % 16 == 0 && (kWinCopy * 4) % 16 == 0, "window layout");
constexpr uint32_t kTmemCols = kAccBufs * kTileN;
constexpr int kBoundSlack = 3;      // the pass-1 bound stops once K..K+3 class maxima are above it
constexpr int kMaxBand = 32;        // wide: boundary candidates rescored per row (one per lane) before falling back

// Two variants.  Narrow (K <= 64): the pass-1 bound is the K-th largest of 128
// column-class maxima (key mod 128); the candidate sub-lists (about 1.3 K per
// row on random data) sit in shared memory and the epilogue warps make the final
// choice in the kernel.  Wide (64 < K <= 128): 256 classes (key tile parity x
// column; pass 1 visits the even tiles, then the odd ones); the sub-lists (about
// 1.4 K per row) sit in global memory and a warp-per-row kernel
// (final_select_kernel) makes the final choice.
// Variants.  kD is the contraction width: 64 for the router's projections, 128
// for the exact-dot oracle selector (q . k at head_dim 128, no position bias).
// A kD = 128 tile is stored as two 128 x 64 sub-tiles (one TMA box and one
// swizzle atom column each), so the K = 128 contraction walks two descriptor
// bases.  With kD = 128 the operand tiles double, so the candidate lists always
// go to global memory and the wide variant stores its class maxima as fp16,
// rounded down (still a lower bound).
template <bool kWide, int kD = 64>
struct TcCfg {
    static_assert(kD == 64 || kD == 128, "contraction width");
    static constexpr int kMaxK = kWide ? 128 : 64;
    static constexpr bool kGlobal = kWide || kD > 64;       // candidate lists in global memory
    static constexpr bool kClsHalf = kWide && kD > 64;      // class maxima as fp16
    static constexpr int kTileB = kTileM * kD * 2;          // bytes of one q' or k' tile
    static constexpr int kStages = kD > 64 ? 3 : (kWide ? 4 : 2);  // k' tile ring
    // sub-list capacity per row and column half (global lists for kD = 128 take
    // more room than the shared-memory lists of the narrow kD = 64 variant)
    static constexpr int kCap = kWide ? 160 : (kD > 64 ? 96 : 80);
    static constexpr int kLimit = kCap - 16;       // past this after a 16-column step: exact fallback
    // shared-memory lists (narrow, kD = 64): kRowStride uint2 per row (both
    // sub-lists and a spare entry for the row's bound and counts; the odd stride
    // spreads banks); the class maxima go through the still empty sub-list area.
    static constexpr int kRowStride = 2 * kCap + 1;
    // global lists: class maxima kClsStride entries per row (wide: 256 classes,
    // odd stride; narrow: 128, stride 2 (mod 32) banks), then the per-row bounds;
    // sub-lists contiguous per row and half, 2 * kTileM * kCap entries per query
    // block.
    static constexpr int kClsStride = kWide ? 2 * kTileN + 1 : kTileN + 2;
    static constexpr size_t kClsBytes = (size_t)kTileM * kClsStride * (kClsHalf ? 2 : 4);
    static constexpr size_t kOffA = 0;
    static constexpr size_t kOffB = kOffA + kTileB;
    static constexpr size_t kOffWin = kOffB + (size_t)kStages * kTileB;
    static constexpr size_t kOffBuf = kOffWin + (size_t)kAccBufs * kWinBytes;
    static constexpr size_t kOffLb = kOffBuf + (kClsBytes + 15) / 16 * 16;  // global lists: bound per row
    static constexpr size_t kBufBytes =
        kGlobal ? (kOffLb - kOffBuf) + (size_t)kTileM * 4 : (size_t)kTileM * kRowStride * sizeof(uint2);
    static constexpr size_t kOffBar = (kOffBuf + kBufBytes + 7) / 8 * 8;
    static constexpr int kNumBars = 2 * kStages + 1 + 2 * kAccBufs + 2;
    static constexpr size_t kOffSlot = kOffBar + (size_t)kNumBars * 8;
    static constexpr size_t kSmemBytes = kOffSlot + 16 + 1024;  // + alignment slack
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    static_assert(kOffB % 1024 == 0 && kTileB % 1024 == 0, "swizzled tiles need 1 KB alignment");
    static_assert(kOffWin % 16 == 0, "bulk copies need 16-byte aligned destinations");
    static_assert(kGlobal || kTileM * 256 <= kStages * kTileB, "output staging fits in the k' ring");
};
constexpr int kWideMaxK = TcCfg<true>::kMaxK;
constexpr int kNarrowMaxK = TcCfg<false>::kMaxK;

constexpr int kSkipMinTiles = 40;  // key tiles from which pass 2 tests the half-tile skip

// ---------------------------------------------------------------- prep kernels

// Per (b, kv head) statistics: the kStatWords words described in router_prep.cuh.
template <int kD>
__global__ void kstats_kernel(const float* __restrict__ kp, int N, uint32_t* __restrict__ stats) {
    const int bg = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    float mabs = 0.f, ss = 0.f;
    bool bad = false;
    if (j < N) {
        const float4* r = reinterpret_cast<const float4*>(kp + ((size_t)bg * N + j) * kD);
#pragma unroll
        for (int c = 0; c < kD / 4; ++c) {
            const float4 x = __ldg(r + c);
            mabs = fmaxf(mabs, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
            ss = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, fmaf(x.w, x.w, ss))));
            bad |= !(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w));
        }
    }
    const float nrm = sqrtf(ss) * 1.0001f;
    uint32_t m1 = __reduce_max_sync(kFull, __float_as_uint(mabs));
    uint32_t m2 = __reduce_max_sync(kFull, __float_as_uint(bad ? 0.f : nrm));
    unsigned b = __reduce_or_sync(kFull, bad ? 1u : 0u);
    if ((threadIdx.x & 31) == 0) {
        atomicMax(stats + kStatWords * bg + 0, m1);
        atomicMax(stats + kStatWords * bg + 1, m2);
        if (b) atomicOr(stats + kStatWords * bg + 2, 1u);
    }
}

// gstats[0] = max |bias| bits, gstats[1] = non-finite flag.
__global__ void bias_stats_kernel(const float* __restrict__ bias, int n, uint32_t* __restrict__ gstats) {
    float m = 0.f;
    bool bad = false;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x) {
        const float x = __ldg(bias + t);
        bad |= !isfinite(x);
        m = fmaxf(m, fabsf(x));
    }
    const uint32_t mm = __reduce_max_sync(kFull, __float_as_uint(m));
    const unsigned b = __reduce_or_sync(kFull, bad ? 1u : 0u);
    if ((threadIdx.x & 31) == 0) {
        atomicMax(gstats + 0, mm);
        if (b) atomicOr(gstats + 1, 1u);
    }
}

// The pos_bias windows of one call, one per tile diagonal d = nqb - 1 - qb + key
// tile: the exact shared-memory image of the tile's window (kWinBytes), so one
// bulk copy brings it in.  Copy s of window d holds, at position y < kWinLen, the
// bias term of offset o = o_max - kTileN * d - y - s (o = i - j + L; offsets
// descend so that ascending positions are ascending key columns): -inf when
// causal and o < L (a key after its query), else pos_bias[clamp(o, 0, 2L - 1)]
// (0 with no pos_bias: the oracle's plain scaled dot products).
__global__ void window_table_kernel(const float* __restrict__ bias, int L, int causal, long long o_max, int ndiag,
                                    float* __restrict__ out) {
    constexpr int kPer = 4 * kWinCopy;
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)ndiag * kPer) return;
    const int d = (int)(t / kPer);
    const int r = (int)(t - (long long)d * kPer);
    const int s = r / kWinCopy, y = r - s * kWinCopy;
    const long long o = o_max - (long long)kTileN * d - y - s;
    float v = 0.f;  // copy padding
    if (y < kWinLen)
        v = (causal && o < L) ? -INFINITY
                              : (bias ? __ldg(bias + (o < 0 ? 0 : (o > 2LL * L - 1 ? 2LL * L - 1 : o))) : 0.f);
    out[t] = v;
}

// Tile diagonals of a call: tile (qb, key tile) uses window nqb - 1 - qb + key tile.
__host__ __device__ constexpr int window_count(int nqb, int tiles_n) { return nqb + tiles_n - 1; }

// Largest bias term of each (tile diagonal d, column half hf, tile row r): the maximum
// over the 64 columns c of that half of the window value of (r, c), u_d[c - r + 127]
// (-inf where every column is causally masked).  Read from the window images: u_d[z]
// is copy 0 at position z for z < kWinLen, copy 3 at z - 3 above.  Pass 2 of the
// selector skips a warp's half tile when no row can reach its threshold there.
__global__ void window_max_kernel(const float* __restrict__ wtab, int ndiag, float* __restrict__ out) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)ndiag * 2 * kTileM) return;
    const int d = (int)(t / (2 * kTileM));
    const int rem = (int)(t - (long long)d * 2 * kTileM);
    const int hf = rem / kTileM, r = rem - hf * kTileM;
    const float* w = wtab + (size_t)d * (4 * kWinCopy);
    float mx = -INFINITY;
    for (int c = 64 * hf; c < 64 * hf + 64; ++c) {
        const int z = c - r + (kTileN - 1);
        const float v = z < kWinLen ? __ldg(w + z) : __ldg(w + 3 * kWinCopy + (z - 3));
        mx = fmaxf(mx, v);
    }
    out[t] = mx;
}

// fp16 copy of k' scaled by the (b, kv head) power of two, one float4 per thread
// (kD / 4 threads per key row), and the norm of each row's conversion error,
// whose maximum goes to stats[kStatWords*bg + 3].  Blocks of 256 threads.
template <int kD>
__global__ void kconvert_kernel(const float* __restrict__ kp, __half* __restrict__ k16, int N,
                                uint32_t* __restrict__ stats) {
    constexpr int kTPR = kD / 4;  // threads per row
    const int bg = blockIdx.y;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = (long long)t < (long long)N * kTPR;  // whole rows share it
    const int e = scale_exponent(__uint_as_float(stats[kStatWords * bg + 0]));
    float ss = 0.f;
    if (live) {
        const size_t off = (size_t)bg * N * kD + (size_t)t * 4;
        const float4 x = __ldg(reinterpret_cast<const float4*>(kp + off));
        const float up = pow2f(e), dn = pow2f(-e);
        __half2 lo = __floats2half2_rn(scale2(x.x, e, up), scale2(x.y, e, up));
        __half2 hi = __floats2half2_rn(scale2(x.z, e, up), scale2(x.w, e, up));
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(k16 + off) = pk;
        // conversion errors in unscaled units (power-of-two scaling and the
        // difference of two values within a factor of 2 are exact)
        const float2 fl = __half22float2(lo), fh = __half22float2(hi);
        const float d0 = scale2(fl.x, -e, dn) - x.x, d1 = scale2(fl.y, -e, dn) - x.y;
        const float d2 = scale2(fh.x, -e, dn) - x.z, d3 = scale2(fh.y, -e, dn) - x.w;
        ss = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, d3 * d3)));
    }
#pragma unroll
    for (int o = 1; o < kTPR; o <<= 1) ss += __shfl_xor_sync(kFull, ss, o);
    // maximum over the block's rows, then one atomic per block (same-address
    // atomics from every warp serialise)
    __shared__ uint32_t wmax[8];
    const uint32_t nrm = live ? __float_as_uint(sqrtf(ss) * 1.0001f) : 0u;
    const uint32_t m = __reduce_max_sync(kFull, nrm);
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t bmax = 0u;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) bmax = max(bmax, wmax[w]);
        if (bmax != 0u) atomicMax(stats + kStatWords * bg + 3, bmax);
    }
}

// Eight threads per query row (kD / 8 values each, coalesced loads and
// stores): scaled fp16 row, epilogue multiplier and error bound.
template <int kD>
// Also rowub[row]: a bound on (approximate score - position bias term) for every key of
// the row: scale |q'| max|k'| + delta with margins for the roundings.
__global__ void __launch_bounds__(256) qprep_kernel(const float* __restrict__ qp, __half* __restrict__ q16,
                                                    float2* __restrict__ rowinfo, float* __restrict__ rowub,
                                                    long long rows, int H, int Hkv, int Nq, float scale,
                                                    const uint32_t* __restrict__ stats,
                                                    const uint32_t* __restrict__ gstats) {
    constexpr int kV4 = kD / 32;  // float4 per thread
    const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int part = threadIdx.x & 7;
    const bool live = row < rows;  // whole 8-lane groups share it
    const long long rr = live ? row : 0;
    const long long bh = rr / Nq;
    const int b = (int)(bh / H);
    const int h = (int)(bh - (long long)b * H);
    const int bg = b * Hkv + h / (H / Hkv);
    const float4* r = reinterpret_cast<const float4*>(qp + rr * kD) + kV4 * part;
    float4 x[kV4];
    float mabs = 0.f, ss = 0.f;
    unsigned bad = 0u;
#pragma unroll
    for (int v = 0; v < kV4; ++v) {
        x[v] = __ldg(r + v);
        mabs = fmaxf(mabs, fmaxf(fmaxf(fabsf(x[v].x), fabsf(x[v].y)), fmaxf(fabsf(x[v].z), fabsf(x[v].w))));
        ss = fmaf(x[v].x, x[v].x, fmaf(x[v].y, x[v].y, fmaf(x[v].z, x[v].z, fmaf(x[v].w, x[v].w, ss))));
        bad |= (isfinite(x[v].x) && isfinite(x[v].y) && isfinite(x[v].z) && isfinite(x[v].w)) ? 0u : 1u;
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        mabs = fmaxf(mabs, __shfl_xor_sync(kFull, mabs, o));
        ss += __shfl_xor_sync(kFull, ss, o);
        bad |= __shfl_xor_sync(kFull, bad, o);
    }
    if (!live) return;
    const int eq = scale_exponent(mabs);
    const float up = pow2f(eq), dn = pow2f(-eq);
    // fp16 copy, and the conversion errors of this part of the row in unscaled
    // units (power-of-two scaling and the difference of two values within a
    // factor of 2 are exact)
    float dd = 0.f;
    uint2 pk[kV4];
#pragma unroll
    for (int v = 0; v < kV4; ++v) {
        const __half2 h0 = __floats2half2_rn(scale2(x[v].x, eq, up), scale2(x[v].y, eq, up));
        const __half2 h1 = __floats2half2_rn(scale2(x[v].z, eq, up), scale2(x[v].w, eq, up));
        pk[v].x = *reinterpret_cast<const uint32_t*>(&h0);
        pk[v].y = *reinterpret_cast<const uint32_t*>(&h1);
        const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
        const float e0 = scale2(f0.x, -eq, dn) - x[v].x, e1 = scale2(f0.y, -eq, dn) - x[v].y;
        const float e2 = scale2(f1.x, -eq, dn) - x[v].z, e3 = scale2(f1.y, -eq, dn) - x[v].w;
        dd = fmaf(e0, e0, fmaf(e1, e1, fmaf(e2, e2, fmaf(e3, e3, dd))));
    }
    uint4* o = reinterpret_cast<uint4*>(q16 + rr * kD + (size_t)part * kV4 * 4);
#pragma unroll
    for (int v = 0; v < kV4; v += 2) o[v / 2] = make_uint4(pk[v].x, pk[v].y, pk[v + 1].x, pk[v + 1].y);
#pragma unroll
    for (int o2 = 1; o2 < 8; o2 <<= 1) dd += __shfl_xor_sync(0xffu << (threadIdx.x & 24), dd, o2);
    if (part != 0) return;
    row_finish<kD>(rr, eq, ss, dd, bad != 0u, bg, scale, stats, gstats, rowinfo, rowub);
}

// ------------------------------------------------------------ selection kernel

struct TcParams {
    const float2* rowinfo;
    const float* bias;
    const float* qp32;
    const float* kp32;
    int32_t* out;
    int* fb_count;
    int32_t* fb_list;
    int* status;
    const float* wtab;  // pos_bias window images, one per tile diagonal (kWinBytes each)
    const float* wmax;  // per diagonal, column half and tile row: the largest window value
    const float* rowub; // per row: bound on |approximate score - bias term|
    // non-null: qp32 holds only the rows computed on demand (warp_canon_q2) from the
    // bf16 query rows q_in and the transposed Wq
    const __nv_bfloat16* q_in;
    const float* wt;
    uint2* lists;  // wide: (score, key) sub-lists, TcCfg::kCap per row and column half
    int* counts;   // wide: sub-list lengths, -1 sends the row to the exact fallback
    int L, H, Hkv, N, K, causal, nqb;
    int Nq, q0;  // query rows per (b, h) and the key-sequence position of row 0
    float scale;
};

// Canonical fp32 score of (query row qrow, key row krow): the fmaf chain over
// d = 0..kD-1 in order, times scale, plus (router) the position-bias term at
// offset i - j.  Key-row loads go out 64 values at a time (one memory round
// trip for kD = 64; the query row is reused and cached).  kQcg: the query row may
// have been written by this kernel (warp_canon_q2), so it is read through L2.
template <int kD = kR, bool kBias = true, bool kQcg = false>
__device__ __forceinline__ float canonical_score(const float* __restrict__ qrow, const float* __restrict__ krow,
                                                 const float* __restrict__ bias, int L, int i, int j,
                                                 float scale) {
    float bv = 0.f;
    if constexpr (kBias) {
        int bi = i - j + L;
        bi = bi < 0 ? 0 : (bi > 2 * L - 1 ? 2 * L - 1 : bi);
        bv = __ldg(bias + bi);
    }
    float acc = 0.f;
#pragma unroll
    for (int c0 = 0; c0 < kD / 4; c0 += 16) {
        float4 bk[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) bk[u] = __ldg(reinterpret_cast<const float4*>(krow) + c0 + u);
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            const float4 a = kQcg ? __ldcg(reinterpret_cast<const float4*>(qrow) + c0 + u)
                                  : __ldg(reinterpret_cast<const float4*>(qrow) + c0 + u);
            acc = fmaf(a.x, bk[u].x, acc);
            acc = fmaf(a.y, bk[u].y, acc);
            acc = fmaf(a.z, bk[u].z, acc);
            acc = fmaf(a.w, bk[u].w, acc);
        }
    }
    if constexpr (kBias) return __fadd_rn(__fmul_rn(acc, scale), bv);
    else return __fmul_rn(acc, scale);
}

// count_ge over every 8-entry chunk of x: slots past a list's end hold -inf and count
// for no finite v.  (Skipping the chunks past the warp's longest list costs a branch
// per chunk, which measured slower than counting them.)
template <int NX>
__device__ __forceinline__ int count_ge_chunks(const float (&x)[NX], float v) {
    int c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int ch = 0; ch < NX / 8; ++ch) {
#pragma unroll
        for (int u = 0; u < 8; ++u) c[u] += x[8 * ch + u] >= v ? 1 : 0;
    }
    return ((c[0] + c[1]) + (c[2] + c[3])) + ((c[4] + c[5]) + (c[6] + c[7]));
}

// Barrier over `count` threads (a multiple of 32) using hardware barrier `id`.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Count of x[q] >= v (eight independent partial counts: no long add chain).
template <int NX>
__device__ __forceinline__ int count_ge(const float (&x)[NX], float v) {
    int c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int q = 0; q < NX; ++q) c[q & 7] += x[q] >= v ? 1 : 0;
    return ((c[0] + c[1]) + (c[2] + c[3])) + ((c[4] + c[5]) + (c[6] + c[7]));
}

// Next probe of a search for the value v where count(x >= v) reaches `target`:
// linear interpolation of the count between (lo, c_lo) and (hi, c_hi), kept in
// the middle 7/8 of the bracket so that every step shrinks it.  On the class
// maxima (spread smoothly between their min and max) it takes fewer steps than
// bisection; correctness never depends on where it probes.
__device__ __forceinline__ float interp_probe(float lo, float hi, int c_lo, int c_hi, float target) {
    const float den = (float)(c_lo - c_hi);
    float t = den > 0.f ? __fdividef((float)c_lo - target, den) : 0.5f;
    t = fminf(fmaxf(t, 0.0625f), 0.9375f);
    return lo + t * (hi - lo);
}

// Class-maximum storage: fp32, or fp16 rounded toward -inf (a smaller value,
// so the K-th largest stays a lower bound on the K-th best score).
__device__ __forceinline__ void cls_put(float* p, float v) { *p = v; }
__device__ __forceinline__ void cls_put(__half* p, float v) { *p = __float2half_rd(v); }
__device__ __forceinline__ float cls_get(const float* p) { return *p; }
__device__ __forceinline__ float cls_get(const __half* p) { return __half2float(*p); }

// A lower bound on the K-th largest class maximum of a row whose maxima are
// spread over G consecutive lanes (kHalfCols per lane, -inf for empty classes):
// bisection on the value until K..K+kBoundSlack maxima are >= lo (or the bracket
// cannot be split).  K distinct keys reach the result, so it is a lower bound on
// the row's K-th best approximate score; -inf when fewer than K are finite.
template <int G>
__device__ __forceinline__ float group_class_bound(const float (&y)[kHalfCols], int K) {
    float lo8[8], hi8[8];
    int nf8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        lo8[u] = INFINITY;
        hi8[u] = -INFINITY;
        nf8[u] = 0;
    }
#pragma unroll
    for (int c = 0; c < kHalfCols; ++c) {
        const bool f = y[c] > -INFINITY;
        nf8[c & 7] += f ? 1 : 0;
        lo8[c & 7] = f ? fminf(lo8[c & 7], y[c]) : lo8[c & 7];
        hi8[c & 7] = fmaxf(hi8[c & 7], y[c]);
    }
    float lo = lo8[0], hi = hi8[0];
    int nfin = nf8[0];
#pragma unroll
    for (int u = 1; u < 8; ++u) {
        lo = fminf(lo, lo8[u]);
        hi = fmaxf(hi, hi8[u]);
        nfin += nf8[u];
    }
#pragma unroll
    for (int o = 1; o < G; o <<= 1) {
        lo = fminf(lo, __shfl_xor_sync(kFull, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(kFull, hi, o));
        nfin += __shfl_xor_sync(kFull, nfin, o);
    }
    bool done = nfin <= K + kBoundSlack;
    int c_lo = nfin, c_hi = 1;  // count(y >= lo), an estimate of count(y >= hi)
    for (int it = 0; it < 32; ++it) {
        if (__all_sync(kFull, done)) break;
        const float mid = interp_probe(lo, hi, c_lo, c_hi, (float)K + 0.5f * kBoundSlack);
        int c = count_ge<kHalfCols>(y, mid);
#pragma unroll
        for (int o = 1; o < G; o <<= 1) c += __shfl_xor_sync(kFull, c, o);
        if (!done) {
            if (!(mid > lo && mid < hi)) {
                done = true;
            } else if (c >= K) {
                lo = mid;
                c_lo = c;
                done = c <= K + kBoundSlack;  // any lo with >= K maxima above is a bound
            } else {
                hi = mid;
                c_hi = c;
            }
        }
    }
    return nfin < K ? -INFINITY : lo;
}

// Candidate append: store (sc, key) at a and advance a by one entry (kStep
// bytes) when sc >= theta (and, in the masked form, col < climit).  The address
// chain only carries the add; the compare is repeated off it, so the compiler
// can compute the next columns' compares ahead.  Shared-memory sub-lists take a
// 32-bit shared address, global ones a 64-bit global address.
template <uint32_t kStep>
__device__ __forceinline__ void append_ge(uint32_t& a, float sc, float theta, uint32_t key) {
    asm volatile("{\n .reg .pred p;\n setp.ge.f32 p, %1, %2;\n"
                 " @p st.shared.v2.b32 [%0], {%1, %3};\n}" :: "r"(a), "f"(sc), "f"(theta), "r"(key));
    a += sc >= theta ? kStep : 0u;
}
template <uint32_t kStep>
__device__ __forceinline__ void append_ge_lt(uint32_t& a, float sc, float theta, uint32_t key, int col,
                                             int climit) {
    asm volatile("{\n .reg .pred p, e;\n setp.ge.f32 p, %1, %2;\n setp.lt.s32 e, %4, %5;\n"
                 " and.pred p, p, e;\n @p st.shared.v2.b32 [%0], {%1, %3};\n}"
                 :: "r"(a), "f"(sc), "f"(theta), "r"(key), "r"(col), "r"(climit));
    a += (sc >= theta && col < climit) ? kStep : 0u;
}
template <uint64_t kStep>
__device__ __forceinline__ void append_ge(uint64_t& a, float sc, float theta, uint32_t key) {
    asm volatile("{\n .reg .pred p;\n setp.ge.f32 p, %1, %2;\n"
                 " @p st.global.v2.b32 [%0], {%1, %3};\n}" :: "l"(a), "f"(sc), "f"(theta), "r"(key));
    a += sc >= theta ? kStep : 0ull;
}
template <uint64_t kStep>
__device__ __forceinline__ void append_ge_lt(uint64_t& a, float sc, float theta, uint32_t key, int col,
                                             int climit) {
    asm volatile("{\n .reg .pred p, e;\n setp.ge.f32 p, %1, %2;\n setp.lt.s32 e, %4, %5;\n"
                 " and.pred p, p, e;\n @p st.global.v2.b32 [%0], {%1, %3};\n}"
                 :: "l"(a), "f"(sc), "f"(theta), "r"(key), "r"(col), "r"(climit));
    a += (sc >= theta && col < climit) ? kStep : 0ull;
}

// Scores of two adjacent columns in one instruction: (acc0, acc1) * (m, m) +
// (b0, b1) with fma.rn.f32x2, each element rounded exactly as fmaf.  mm holds
// m in both halves.
__device__ __forceinline__ float2 score2(uint32_t acc0, uint32_t acc1, uint64_t mm, float b0, float b1) {
    float2 d;
    asm("{\n .reg .b64 ra, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rc, {%5, %6};\n"
        " fma.rn.f32x2 rd, ra, %4, rc;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y) : "r"(acc0), "r"(acc1), "l"(mm), "f"(b0), "f"(b1));
    return d;
}

// Scores one 64-column half tile in 16-column chunks, software-pipelined:
// chunk h + 1's accumulator columns (tcgen05.ld) and pos_bias terms (ld.shared
// from wsrc upwards, x..w = columns c..c+3) are in flight while chunk h is
// scored by fn(h, v, bw).
// The accumulator and the window buffer are released on `tempty` after the last
// chunk has been scored: the next MMA into this accumulator and the bulk copy of
// the next window into this buffer start as soon as `tempty` completes.  Every
// accumulator load of the half tile has completed at the release (tcgen05.wait::ld
// precedes each chunk's use, then tcgen05.fence::before_thread_sync); one word of
// every 16-byte window load is OR-ed into `dep`, the warp reduces it (each lane
// waits for its own loads) and the arrive's address depends on the result, so no
// read of this tile can still be in flight at the release.  (A release issued
// before the last chunk was scored let the next tile's MMA and window copy land
// under the last chunk's reads on B200.)
template <typename Fn>
__device__ __forceinline__ void score_half_tile(uint32_t taddr, uint32_t wsrc, uint64_t* tempty, int lane, Fn&& fn) {
    constexpr int kC = 16, kNC = kHalfCols / kC;
    uint32_t v[2][kC];
    float4 bw[2][kC / 4];
    uint32_t dep = 0u;
    tmem_ld16(taddr, v[0]);
#pragma unroll
    for (int q = 0; q < kC / 4; ++q) bw[0][q] = lds_f4(wsrc + 16u * (uint32_t)q);
#pragma unroll
    for (int h = 0; h < kNC; ++h) {
        tmem_wait_ld();
        reg_fence(v[h & 1]);
        if (h + 1 < kNC) {
            tmem_ld16(taddr + (uint32_t)(kC * (h + 1)), v[(h + 1) & 1]);
#pragma unroll
            for (int q = 0; q < kC / 4; ++q) bw[(h + 1) & 1][q] = lds_f4(wsrc + 4u * (uint32_t)(kC * (h + 1) + 4 * q));
        }
        fn(h, v[h & 1], bw[h & 1]);
#pragma unroll
        for (int q = 0; q < kC / 4; ++q) dep |= __float_as_uint(bw[h & 1][q].x);
    }
    tc_fence_before();
    dep = __reduce_or_sync(kFull, dep);
    if (lane == 0) mbar_arrive_after(tempty, dep);
}

template <bool kWide, int kD = 64, bool kSkip = false>
__global__ void __launch_bounds__(kThreads, 1)
router_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const TcParams p) {
    using Cfg = TcCfg<kWide, kD>;
    constexpr int kStages = Cfg::kStages;
    constexpr int kTB = Cfg::kTileB;
    constexpr bool kGlobal = Cfg::kGlobal;
    using ClsT = std::conditional_t<Cfg::kClsHalf, __half, float>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sA = smem + Cfg::kOffA;
    uint8_t* sB = smem + Cfg::kOffB;
    float* win = reinterpret_cast<float*>(smem + Cfg::kOffWin);
    // shared-memory lists, or class maxima and bounds (see TcCfg)
    [[maybe_unused]] uint2* buf = reinterpret_cast<uint2*>(smem + Cfg::kOffBuf);
    [[maybe_unused]] ClsT* cls = reinterpret_cast<ClsT*>(smem + Cfg::kOffBuf);
    [[maybe_unused]] float* lbw = reinterpret_cast<float*>(smem + Cfg::kOffLb);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* full = bars;
    uint64_t* empty = bars + kStages;
    uint64_t* afull = bars + 2 * kStages;
    uint64_t* tfull = afull + 1;
    uint64_t* tempty = tfull + kAccBufs;
    uint64_t* mdone = tempty + kAccBufs;
    uint64_t* wtbar = mdone + 1;  // narrow, on-demand q' rows: transposed Wq in shared memory
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffSlot);

    const int N = p.N, H = p.H, Hkv = p.Hkv, Nq = p.Nq;
    const int BH = gridDim.x / p.nqb;
    const int order = blockIdx.x / BH;
    const int bh = blockIdx.x - order * BH;
    const int qb = p.causal ? (p.nqb - 1 - order) : order;
    const int b = bh / H;
    const int h = bh - b * H;
    const int g = h / (H / Hkv);
    const int i0 = qb * kTileM;     // first query row of the block (local index)
    const int i0g = p.q0 + i0;      // its position in the key sequence
    const int jend = p.causal ? min(N, i0g + kTileM) : N;
    const int T = (jend + kTileN - 1) / kTileN;  // key tiles per pass
    const int T2 = 2 * T;                          // two passes over the same key tiles
    // Key tile of step t.  Pass 2 (t >= T) walks the tiles in order, and so does
    // pass 1 of the narrow selection; the wide selection's pass 1 takes the even
    // tiles first and the odd ones after, so each parity has its own class maxima.
    const int Te = (T + 1) >> 1;
    auto tile_of = [T, Te](int t) -> int {
        if (t >= T) return t - T;
        if constexpr (kWide) return t < Te ? 2 * t : 2 * (t - Te) + 1;
        return t;
    };
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        mbar_init(afull, 1);
        for (int s = 0; s < kAccBufs; ++s) {
            mbar_init(tfull + s, 2);  // MMA commit + the window's bulk copy
            mbar_init(tempty + s, kEpiWarps);
        }
        mbar_init(mdone, 1);
        mbar_init(wtbar, 2);  // the two halves of Wq transposed (MMA warp, window warp)
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            bool ok = true;
            // a tile is kD / 64 boxes of 128 rows x 64 columns (one 16 KB swizzle atom column each)
            mbar_arrive_expect_tx(afull, kTB);
#pragma unroll
            for (int h = 0; h < kD / 64; ++h) tma_load_2d(sA + h * 16384, &tmA, afull, 64 * h, bh * Nq + i0);
            const int krow0 = (b * Hkv + g) * N;
            int issued = 0;
            for (int t = 0; t < T2; ++t) {
                const int s = t % kStages;
                if (t >= kStages) ok = mbar_wait(empty + s, ((t / kStages) - 1) & 1);
                if (!ok) break;
                mbar_arrive_expect_tx(full + s, kTB);
#pragma unroll
                for (int h = 0; h < kD / 64; ++h)
                    tma_load_2d(sB + (size_t)s * kTB + h * 16384, &tmB, full + s, 64 * h, krow0 + tile_of(t) * kTileN);
                issued = t + 1;
            }
            // the loads of the last stages are never waited on by a refill: make
            // sure they have landed before the CTA can retire
            for (int t = max(0, issued - kStages); t < issued; ++t) mbar_wait(full + t % kStages, (t / kStages) & 1);
            mbar_wait(afull, 0);
            if (!ok) atomicOr(p.status, 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(0u, kTileM, kTileN);
            bool ok = mbar_wait(afull, 0);
            for (int t = 0; t < T2 && ok; ++t) {
                const int s = t % kStages;
                const int ab = t % kAccBufs;
                ok = mbar_wait(full + s, (t / kStages) & 1);
                if (ok && t >= kAccBufs) ok = mbar_wait(tempty + ab, ((t / kAccBufs) - 1) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(ab * kTileN);
#pragma unroll
                for (int k = 0; k < kD / 16; ++k) {
                    // 16 columns per MMA; a new 64-column atom column every 4
                    const uint64_t ad = umma_desc_sw128(sA + (k >> 2) * 16384) + 2u * (k & 3);
                    const uint64_t bd = umma_desc_sw128(sB + (size_t)s * kTB + (k >> 2) * 16384) + 2u * (k & 3);
                    mma_f16(d, ad, bd, idesc, k > 0 ? 1u : 0u);
                }
                mma_commit(empty + s);
                mma_commit(tfull + ab);
            }
            mma_commit(mdone);  // completes once every MMA issued above has finished
            mbar_wait(mdone, 0);
            if constexpr (!kGlobal) {
                // on-demand q' rows: d = 0..63 of Wq transposed into the query tile, idle
                // now that every MMA has completed
                if (ok && p.q_in != nullptr) {
                    mbar_arrive_expect_tx(wtbar, 16384);
                    bulk_load(sA, p.wt, 16384, wtbar);
                }
            }
            if (!ok) atomicOr(p.status, 2);
        }
    } else if (warp == 2) {
        // ------------------------------------------------ window loads
        // The pos_bias window of step t goes to window buffer t % kAccBufs once the
        // accumulator of that index is free (every epilogue warp is done with
        // both), as one bulk copy of its precomputed image that completes on the
        // accumulator's tfull barrier (its second arrival, after the MMA commit).
        if (lane == 0) {
            const float* wbase = p.wtab + (size_t)(p.nqb - 1 - qb) * (4 * kWinCopy);
            bool ok = true;
            int issued = 0;
            for (int t = 0; t < T2; ++t) {
                const int ab = t % kAccBufs;
                if (t >= kAccBufs) ok = mbar_wait(tempty + ab, ((t / kAccBufs) - 1) & 1);
                if (!ok) break;
                mbar_arrive_expect_tx(tfull + ab, kWinBytes);
                bulk_load(win + (size_t)ab * (kWinBytes / 4), wbase + (size_t)tile_of(t) * (4 * kWinCopy), kWinBytes,
                          tfull + ab);
                issued = t + 1;
            }
            // copies the epilogue never waited for (error path) land before the CTA
            // retires: their barrier phases complete, or the bounded waits run out
            // long after the bytes have arrived
            if (!ok)
                for (int t = max(0, issued - kAccBufs); t < issued; ++t)
                    mbar_wait(tfull + t % kAccBufs, (t / kAccBufs) & 1);
            if constexpr (!kGlobal) {
                // on-demand q' rows: d = 64..127 of Wq transposed into the window
                // buffers once every epilogue warp has released the last of them
                if (ok && p.q_in != nullptr) {
                    for (int t = max(0, T2 - kAccBufs); t < T2 && ok; ++t)
                        ok = mbar_wait(tempty + t % kAccBufs, (t / kAccBufs) & 1);
                    if (ok) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        mbar_arrive_expect_tx(wtbar, 16384);
                        bulk_load(win, p.wt + 4096, 16384, wtbar);
                    }
                }
            }
            if (!ok) atomicOr(p.status, 8);
        }
    } else {
        // ------------------------------------------------ epilogue: scoring + selection
        // Eight warps: warp (quadrant qd, half hf) owns TMEM lanes 32*qd.. (query
        // rows) and accumulator columns 64*hf.. of every tile; each row is served
        // by two threads, one per column half, with one candidate sub-list each.
        const int ew = warp - kCtlWarps;     // 0..7
        const int qd = warp & 3;             // TMEM lane quadrant this warp may access
        const int hf = ew >> 2;              // column half
        const int r0 = qd * 32;
        const int row = r0 + lane;
        const int i = i0 + row;              // local query row
        const int K = p.K;
        const int cbase = hf * kHalfCols;    // first tile column of this thread
        const uint32_t pair_bar = 1u + (uint32_t)qd;  // named barrier of the quadrant's two warps
        float m = 0.f, delta = 0.f;
        bool fb = i >= Nq;  // rows to skip (inactive) or to recompute exactly
        if (i < Nq) {
            const float2 ri = p.rowinfo[(size_t)bh * Nq + i];
            m = ri.x;
            delta = ri.y;
            if (!(m == m)) fb = true;
        }
        const uint64_t mm = ((uint64_t)__float_as_uint(m) << 32) | __float_as_uint(m);  // (m, m)
        // The window holds u[z], z = col - row + 127 (the bias term of column col
        // for this row), copy s holding u[s ..].  Columns cbase + cl .. + 3 (cl a
        // multiple of 4) are copy s4 = 3 - (row & 3) at position
        // cbase + cl - (row - (row & 3)) + 124, in column order.
        const int s4 = 3 - (lane & 3);
        const uint32_t wrd_s =
            smem_u32(win) + 4u * (uint32_t)(s4 * kWinCopy + cbase - (row - (lane & 3)) + (kTileN - 4));
        const int lim = p.causal ? min(N, p.q0 + i + 1) : N;  // keys j < lim are eligible
        bool ok = true;

        // Tile prologue shared by both passes: wait for the tile's accumulator and
        // pos_bias window (one barrier).  Returns false if the bounded wait expired.
        auto tile_prologue = [&](int t) -> bool {
            const bool got = mbar_wait(tfull + t % kAccBufs, (uint32_t)(t / kAccBufs) & 1u);
            if (!__all_sync(kFull, got)) return false;
            tc_fence_after();
            return true;
        };

        // ---------------- pass 1: maximum score per column class (key index mod 128)
        float cm[kHalfCols];
#pragma unroll
        for (int c = 0; c < kHalfCols; ++c) cm[c] = -INFINITY;
        for (int t = 0; t < T && ok; ++t) {
            const int j0 = tile_of(t) * kTileN;
            const int ab = t % kAccBufs;
            if (!tile_prologue(t)) {
                ok = false;
                break;
            }
            const uint32_t taddr = tmem + ((uint32_t)r0 << 16) + (uint32_t)(ab * kTileN + cbase);
            const uint32_t mycopy_s = wrd_s + (uint32_t)(ab * kWinBytes);
            // columns past the last key need the explicit mask (the tile reads on
            // into the next head's keys); causally masked keys score -inf anyway
            const bool full_tile = j0 + cbase + kHalfCols <= N;
            const int climit = lim - j0 - cbase;  // local columns c < climit are eligible
            if (full_tile) {
                score_half_tile(taddr, mycopy_s, tempty + ab, lane,
                                [&](int h, const uint32_t (&v)[16], const float4 (&bw)[4]) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int c = 16 * h + 4 * q;
                        const float2 s01 = score2(v[4 * q + 0], v[4 * q + 1], mm, bw[q].x, bw[q].y);
                        const float2 s23 = score2(v[4 * q + 2], v[4 * q + 3], mm, bw[q].z, bw[q].w);
                        cm[c + 0] = fmaxf(cm[c + 0], s01.x);
                        cm[c + 1] = fmaxf(cm[c + 1], s01.y);
                        cm[c + 2] = fmaxf(cm[c + 2], s23.x);
                        cm[c + 3] = fmaxf(cm[c + 3], s23.y);
                    }
                });
            } else {
                score_half_tile(taddr, mycopy_s, tempty + ab, lane,
                                [&](int h, const uint32_t (&v)[16], const float4 (&bw)[4]) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int c = 16 * h + 4 * q;
                        const float2 s01 = score2(v[4 * q + 0], v[4 * q + 1], mm, bw[q].x, bw[q].y);
                        const float2 s23 = score2(v[4 * q + 2], v[4 * q + 3], mm, bw[q].z, bw[q].w);
                        const float s4v[4] = {s01.x, s01.y, s23.x, s23.y};
#pragma unroll
                        for (int d = 0; d < 4; ++d) {
                            const float sc = s4v[d];
                            cm[c + d] = fmaxf(cm[c + d], c + d < climit ? sc : -INFINITY);
                        }
                    }
                });
            }
            if constexpr (kWide) {
                if (t == Te - 1) {
                    // even tiles done: their class maxima go to shared memory
                    ClsT* crow = cls + row * Cfg::kClsStride + hf * kHalfCols;
#pragma unroll
                    for (int c = 0; c < kHalfCols; ++c) {
                        cls_put(crow + c, cm[c]);
                        cm[c] = -INFINITY;
                    }
                }
            }
        }

        // End of pass 1: a group of lanes per row bounds the row's class maxima
        // (group_class_bound): every exact top-K key scores at least the bound -
        // 2*delta.
        [[maybe_unused]] uint2* rowbuf = buf + (size_t)row * Cfg::kRowStride;  // narrow
        [[maybe_unused]] uint2* sub = rowbuf + hf * Cfg::kCap;  // narrow: this thread's sub-list
        float lb = -INFINITY;
        if constexpr (!kWide && kGlobal) {
            // 128 maxima, 64 per column half, exchanged through the class-maxima
            // area: lanes 2r and 2r+1 of warp hf take row r0 + 16*hf + r, one half each
            ClsT* crow = cls + row * Cfg::kClsStride + hf * kHalfCols;
#pragma unroll
            for (int c = 0; c < kHalfCols; ++c) cls_put(crow + c, cm[c]);
            named_bar_sync(pair_bar, 64);
            const int brow = r0 + 16 * hf + (lane >> 1);
            const int bhalf = lane & 1;
            const ClsT* src = cls + brow * Cfg::kClsStride + bhalf * kHalfCols;
            float y[kHalfCols];
            // rotated by one for the odd lane: with a row stride of 2 (mod 32) banks
            // the warp's 32 reads hit 32 banks
#pragma unroll
            for (int c = 0; c < kHalfCols; ++c) y[c] = cls_get(src + ((c + bhalf) & (kHalfCols - 1)));
            const float lbv = group_class_bound<2>(y, K);
            if (bhalf == 0) lbw[brow] = lbv;
            named_bar_sync(pair_bar, 64);
            lb = lbw[row];
        } else if constexpr (!kWide) {
            // 128 maxima, 64 per column half, exchanged through the still empty
            // sub-lists: lanes 2r and 2r+1 of warp hf take row r0 + 16*hf + r, one
            // half each; the bound goes back through the row's spare entry
            float* xch = reinterpret_cast<float*>(sub);
#pragma unroll
            for (int c = 0; c < kHalfCols; ++c) xch[c] = cm[c];
            named_bar_sync(pair_bar, 64);
            const int brow = r0 + 16 * hf + (lane >> 1);
            const int bhalf = lane & 1;
            const float* bcls = reinterpret_cast<const float*>(buf + (size_t)brow * Cfg::kRowStride + bhalf * Cfg::kCap);
            float y[kHalfCols];
#pragma unroll
            for (int c = 0; c < kHalfCols; ++c) y[c] = bcls[c ^ bhalf];  // the pair reads different banks
            const float lbv = group_class_bound<2>(y, K);
            if (bhalf == 0) buf[(size_t)brow * Cfg::kRowStride + (Cfg::kRowStride - 1)].x = __float_as_uint(lbv);
            named_bar_sync(pair_bar, 64);  // bounds published; class maxima read before sub-lists are written
            lb = __uint_as_float(rowbuf[Cfg::kRowStride - 1].x);
        } else {
            // 256 maxima (even/odd tiles x two column halves, 64 each; the even ones
            // are already in shared memory); four lanes per row, the quadrant's 32
            // rows in two batches of 16
            ClsT* crow = cls + row * Cfg::kClsStride + kTileN + hf * kHalfCols;
#pragma unroll
            for (int c = 0; c < kHalfCols; ++c) cls_put(crow + c, cm[c]);
            named_bar_sync(pair_bar, 64);
#pragma unroll 1
            for (int bt = 0; bt < 2; ++bt) {
                const int brow = r0 + 16 * bt + 8 * hf + (lane >> 2);
                const int t4 = lane & 3;
                const ClsT* src = cls + brow * Cfg::kClsStride + t4 * kHalfCols;
                float y[kHalfCols];
                // rotated by 8 per lane of the group: the warp's 32 fp32 reads hit 32 banks
#pragma unroll
                for (int c = 0; c < kHalfCols; ++c) y[c] = cls_get(src + ((c + 8 * t4) & (kHalfCols - 1)));
                const float lbv = group_class_bound<4>(y, K);
                if (t4 == 0) lbw[brow] = lbv;
            }
            named_bar_sync(pair_bar, 64);
            lb = lbw[row];
        }
        float theta = __int_as_float(0x7fc00000);  // NaN admits nothing
        if (ok && !fb) {
            // fewer than K eligible keys: admit every finite score (masked keys are -inf)
            theta = lb == -INFINITY ? -FLT_MAX : lb - (2.f * delta + fabsf(lb) * kTwoPowM22);
        }

        // ---------------- pass 2: collect candidates s >= theta into the sub-list
        // (narrow: shared memory; wide: global memory, contiguous per row and half)
        using Addr = std::conditional_t<kGlobal, uint64_t, uint32_t>;
        constexpr int kLimit = Cfg::kLimit;
        constexpr Addr kStep = 8;  // bytes per entry
        Addr list_base;
        if constexpr (kGlobal)
            list_base = (uint64_t)__cvta_generic_to_global(
                p.lists + ((size_t)bh * p.nqb + qb) * (2 * kTileM * (size_t)Cfg::kCap) + (size_t)(2 * row + hf) * Cfg::kCap);
        else
            list_base = smem_u32(sub);
        int cnt = 0;
        // Exact skip: every approximate score of this row in a half tile is at most
        // cub + (the half tile's largest bias term for this row); when that is below
        // theta for every row of the warp, the half tile holds no candidate and is
        // released without being read.  (Rows without a finite theta append nothing.)
        // Only query blocks with kSkipMinTiles key tiles or more test it (and only the
        // kSkip build of the kernel, launched when the keys reach that many tiles): the
        // K-th best score of a shorter row sits lower among its scores and the test
        // rarely pays (measured at N = 4096: ~90 cycles per tile, almost no skips).
        const bool try_skip = kSkip && T >= kSkipMinTiles;  // CTA-uniform
        const float cub = (i < Nq && try_skip) ? p.rowub[(size_t)bh * Nq + i] : INFINITY;
        const float* wmax_row = p.wmax + ((size_t)(p.nqb - 1 - qb) * 2 + hf) * kTileM + row;
        float wm_next = try_skip ? __ldg(wmax_row) : 0.f;
        for (int t = T; t < T2 && ok; ++t) {
            const int j0 = (t - T) * kTileN;
            const int ab = t % kAccBufs;
            const float wm = wm_next;
            if (try_skip && t + 1 < T2) wm_next = __ldg(wmax_row + (size_t)(t + 1 - T) * (2 * kTileM));
            if (!tile_prologue(t)) {
                ok = false;
                break;
            }
            if (try_skip) {
                float ub = cub + wm;
                ub += fabsf(ub) * kTwoPowM22;  // the rounding of the sum
                const bool need = theta == theta && !(ub < theta);
                if (!__any_sync(kFull, need)) {
                    tc_fence_before();
                    if (lane == 0) mbar_arrive(tempty + ab);
                    continue;
                }
            }
            const uint32_t taddr = tmem + ((uint32_t)r0 << 16) + (uint32_t)(ab * kTileN + cbase);
            const uint32_t mycopy_s = wrd_s + (uint32_t)(ab * kWinBytes);
            const bool full_tile = j0 + cbase + kHalfCols <= N;
            const int climit = lim - j0 - cbase;
            const uint32_t jb = (uint32_t)(j0 + cbase);
            // Write address and an explicitly predicated store: the per-column
            // append costs one store and one add.
            const Addr sub_s = list_base;
            Addr waddr = sub_s + kStep * (uint32_t)cnt;
            // After every 16 columns: a sub-list that could overflow during the next
            // 16 sends its row to the exact fallback (kLimit = capacity - 16).
            auto overflow_check = [&]() {
                if ((int)((waddr - sub_s) / kStep) > kLimit) {
                    fb = true;
                    theta = __int_as_float(0x7fc00000);
                    waddr = sub_s;
                }
            };
            if (full_tile) {
                score_half_tile(taddr, mycopy_s, tempty + ab, lane,
                                [&](int h, const uint32_t (&v)[16], const float4 (&bw)[4]) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int c = 16 * h + 4 * q;
                        const float b4[4] = {bw[q].x, bw[q].y, bw[q].z, bw[q].w};
#pragma unroll
                        for (int d = 0; d < 4; ++d) {
                            // scalar FMAs here: the packed form measured slower in this loop
                            const float sc = fmaf(__uint_as_float(v[4 * q + d]), m, b4[d]);
                            append_ge<kStep>(waddr, sc, theta, jb + (uint32_t)(c + d));
                        }
                    }
                    overflow_check();
                });
            } else {
                score_half_tile(taddr, mycopy_s, tempty + ab, lane,
                                [&](int h, const uint32_t (&v)[16], const float4 (&bw)[4]) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int c = 16 * h + 4 * q;
                        const float b4[4] = {bw[q].x, bw[q].y, bw[q].z, bw[q].w};
#pragma unroll
                        for (int d = 0; d < 4; ++d) {
                            // scalar FMAs here: the packed form measured slower in this loop
                            const float sc = fmaf(__uint_as_float(v[4 * q + d]), m, b4[d]);
                            append_ge_lt<kStep>(waddr, sc, theta, jb + (uint32_t)(c + d), c + d, climit);
                        }
                    }
                    overflow_check();
                });
            }
            cnt = (int)((waddr - sub_s) / kStep);
        }
        if (!ok) atomicOr(p.status, 4);

        if constexpr (kGlobal) {
            // final_select_kernel finishes the row from its two lists
            if (ok && i < Nq) p.counts[((size_t)bh * Nq + i) * 2 + hf] = fb ? -1 : cnt;
        } else {
            // ---------------------------------------------- per-row final selection
            // Publish both sub-list counts (-1: exact fallback); then the lane pair
            // (2r, 2r+1) of warp hf finishes row r0 + 16*hf + r, each lane owning one
            // sub-list (both are in ascending key order).
            //  1. bisection on the approximate scores from [lb, max] until exactly K
            //     are >= lo; x_K = min{s >= lo}, x_K1 = max{s < lo}.  Entries above
            //     U = x_K1 + 2*delta are certainly in the exact top K, entries below
            //     W = x_K - 2*delta certainly not (with a bracket [lo, hi] instead
            //     when the scores do not split: U = hi + 2*delta, W = lo - 2*delta).
            //  2. entries in [W, U] (usually none) are rescored with the canonical
            //     fp32 formula and the best K - #(s > U) of them by (score desc,
            //     key asc) are kept.
            //  3. each lane compacts its kept keys in place; lane 2r merges the two
            //     lists from the front, lane 2r+1 from the back, into the output row.
            // A row's two counts go to the .y word of its spare list entry (.x holds
            // the bound), 16 bits per column half.
            reinterpret_cast<int16_t*>(&rowbuf[Cfg::kRowStride - 1].y)[hf] = (int16_t)(fb ? -1 : cnt);
            named_bar_sync(pair_bar, 64);
            {
                const int frow = r0 + 16 * hf + (lane >> 1);
                const int fh = lane & 1;
                const int fi = i0 + frow;
                const bool active = ok && fi < Nq;
                uint2* frowbuf = buf + (size_t)frow * Cfg::kRowStride;
                const int16_t* fmeta = reinterpret_cast<const int16_t*>(&frowbuf[Cfg::kRowStride - 1].y);
                const int ca = fmeta[0], cb = fmeta[1];
                uint2* own = frowbuf + fh * Cfg::kCap;
                const int nown = fh ? cb : ca;
                bool to_fallback = active && (ca < 0 || cb < 0);
                bool work = active && !to_fallback;
                const int tot = ca + cb;
                const bool all_in = tot <= K;
                const size_t orow_id = (size_t)bh * Nq + (size_t)(fi < Nq ? fi : 0);
                float fdelta = 0.f, lo = 0.f;
                if (work) {
                    fdelta = p.rowinfo[orow_id].y;
                    lo = __uint_as_float(frowbuf[Cfg::kRowStride - 1].x);
                }
                const uint32_t own_s = smem_u32(own);
                // Slots past a sub-list's end hold -inf and change no count or extremum
                // below (lo, U and W are finite whenever the row has more than K
                // candidates).  The loads and the longer loops stop after the warp's
                // longest list (nch 8-slot chunks, a branch per chunk); the bisection
                // counts and the maximum take every slot, which measured faster than the
                // branches.
                const int nch = (int)((__reduce_max_sync(kFull, work ? (unsigned)nown : 0u) + 7u) >> 3);
                float x[Cfg::kCap];
    #pragma unroll
                for (int ch = 0; ch < Cfg::kCap / 8; ++ch) {
    #pragma unroll
                    for (int u = 0; u < 8; ++u) x[8 * ch + u] = -INFINITY;
                    if (ch < nch) {
    #pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const int q = 8 * ch + u;
                            x[q] = lds_f32_or(own_s + 8u * q, work && q < nown, -INFINITY);
                        }
                    }
                }

                // 1. split at the K-th best approximate score
                float hi8[8];
    #pragma unroll
                for (int u = 0; u < 8; ++u) hi8[u] = -INFINITY;
    #pragma unroll
                for (int ch = 0; ch < Cfg::kCap / 8; ++ch) {
    #pragma unroll
                    for (int u = 0; u < 8; ++u) hi8[u] = fmaxf(hi8[u], x[8 * ch + u]);
                }
                float hi = fmaxf(fmaxf(fmaxf(hi8[0], hi8[1]), fmaxf(hi8[2], hi8[3])),
                                 fmaxf(fmaxf(hi8[4], hi8[5]), fmaxf(hi8[6], hi8[7])));
                hi = fmaxf(hi, __shfl_xor_sync(kFull, hi, 1));
                int cnt_lo = count_ge_chunks<Cfg::kCap>(x, lo);
                cnt_lo += __shfl_xor_sync(kFull, cnt_lo, 1);
                if (work && !all_in && cnt_lo < K) {
                    to_fallback = true;  // cannot happen: lb is reached by K candidates
                    work = false;
                }
                // Stop at an exact split (K entries >= lo) or once the bracket is within
                // 4 delta: the boundary band then holds the few near-tied entries and the
                // canonical rescoring below decides them.
                bool done = !work || all_in || cnt_lo == K || hi - lo <= 4.f * fdelta;
                // (plain bisection: the candidates bunch up near lb, where interpolation
                // on the count probes badly)
                for (int it = 0; it < 40; ++it) {
                    if (__all_sync(kFull, done)) break;
                    const float mid = lo + 0.5f * (hi - lo);
                    int c = count_ge_chunks<Cfg::kCap>(x, mid);
                    c += __shfl_xor_sync(kFull, c, 1);
                    if (!done) {
                        if (!(mid > lo && mid < hi)) {
                            done = true;
                        } else if (c >= K) {
                            lo = mid;
                            cnt_lo = c;
                            done = c == K || hi - lo <= 4.f * fdelta;
                        } else {
                            hi = mid;
                            done = hi - lo <= 4.f * fdelta;
                        }
                    }
                }
                float kmin8[8], kmax8[8];
    #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    kmin8[u] = INFINITY;
                    kmax8[u] = -INFINITY;
                }
    #pragma unroll
                for (int ch = 0; ch < Cfg::kCap / 8; ++ch) {
                    if (ch < nch) {
    #pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const float xq = x[8 * ch + u];
                            const bool ge = xq >= lo;
                            kmin8[u] = ge ? fminf(kmin8[u], xq) : kmin8[u];
                            kmax8[u] = ge ? kmax8[u] : fmaxf(kmax8[u], xq);
                        }
                    }
                }
                float xk = kmin8[0], xk1 = kmax8[0];
    #pragma unroll
                for (int u = 1; u < 8; ++u) {
                    xk = fminf(xk, kmin8[u]);
                    xk1 = fmaxf(xk1, kmax8[u]);
                }
                xk = fminf(xk, __shfl_xor_sync(kFull, xk, 1));
                xk1 = fmaxf(xk1, __shfl_xor_sync(kFull, xk1, 1));
                float U = -INFINITY, W = INFINITY;  // all_in: keep every entry, empty band
                if (work && !all_in) {
                    const bool split = cnt_lo == K && xk1 > -INFINITY;
                    const float top = split ? xk1 : hi;
                    const float bot = split ? xk : lo;
                    const float sl = fmaxf(fabsf(top), fabsf(bot));
                    const float m2 = 2.f * fdelta + (sl + 2.f * fdelta) * kTwoPowM22;
                    U = top + m2;
                    W = bot - m2;
                }
                int n_in = 0, own_nb = 0;
                {
                    int ni8[8] = {0, 0, 0, 0, 0, 0, 0, 0}, nb8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    #pragma unroll
                    for (int ch = 0; ch < Cfg::kCap / 8; ++ch) {
                        if (ch < nch) {
    #pragma unroll
                            for (int u = 0; u < 8; ++u) {
                                const float xq = x[8 * ch + u];
                                ni8[u] += xq > U ? 1 : 0;
                                nb8[u] += (xq >= W && xq <= U) ? 1 : 0;
                            }
                        }
                    }
    #pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        n_in += ni8[u];
                        own_nb += nb8[u];
                    }
                }
                n_in += __shfl_xor_sync(kFull, n_in, 1);
                const int oth_nb = __shfl_xor_sync(kFull, own_nb, 1);
                const int need = K - n_in;
                const bool rescore = work && !all_in && own_nb + oth_nb != need;
                if (p.q_in != nullptr) {
                    // canonical q' of the rows that rescore or go to the exact selector,
                    // one row at a time by the whole warp
                    unsigned pend = __ballot_sync(kFull, (rescore || to_fallback) && fh == 0);
                    if (pend != 0u && !__all_sync(kFull, mbar_wait(wtbar, 0u))) {
                        if (lane == 0) atomicOr(p.status, 16);
                        pend = 0u;
                    }
                    while (pend != 0u) {  // two rows per pass over the weights
                        const int s0 = __ffs(pend) - 1;
                        pend &= pend - 1u;
                        const int s1 = pend != 0u ? __ffs(pend) - 1 : s0;
                        pend &= pend - 1u;
                        const unsigned long long r0 = __shfl_sync(kFull, (unsigned long long)orow_id, s0);
                        const unsigned long long r1 = __shfl_sync(kFull, (unsigned long long)orow_id, s1);
                        float* qp = const_cast<float*>(p.qp32);
                        warp_canon_q2(p.q_in + r0 * 128, p.q_in + r1 * 128, reinterpret_cast<const float*>(sA),
                                           win, qp + r0 * kR, s1 != s0 ? qp + r1 * kR : nullptr, lane);
                    }
                    __syncwarp();
                }

                // 2. canonical rescoring of the boundary band, in place: a band entry's
                // score word becomes the order key of its canonical score; bm marks the
                // band entries of this lane's sub-list, sm the ones selected
                constexpr int kMaskWords = (Cfg::kCap + 31) / 32;
                uint32_t bm[kMaskWords], sm[kMaskWords];
    #pragma unroll
                for (int w = 0; w < kMaskWords; ++w) {
                    bm[w] = 0u;
                    sm[w] = 0u;
                }
                if (rescore) {
    #pragma unroll
                    for (int ch = 0; ch < Cfg::kCap / 8; ++ch) {
                        if (ch < nch) {
    #pragma unroll
                            for (int u = 0; u < 8; ++u) {
                                const int q = 8 * ch + u;
                                bm[q >> 5] |= (x[q] >= W && x[q] <= U) ? 1u << (q & 31) : 0u;
                            }
                        }
                    }
                    const float* qrow = p.qp32 + orow_id * kR;
                    const float* kbase = p.kp32 + (size_t)(b * Hkv + g) * N * kR;
    #pragma unroll
                    for (int w = 0; w < kMaskWords; ++w) {
                        for (uint32_t m = bm[w]; m != 0u; m &= m - 1u) {
                            const int q = 32 * w + __ffs(m) - 1;
                            const int jj = (int)lds_u32(own_s + 8u * q + 4u);
                            const float ex = canonical_score<kR, true, true>(qrow, kbase + (size_t)jj * kR, p.bias,
                                                                             p.L, p.q0 + fi, jj, p.scale);
                            sts_f32(own_s + 8u * q, __uint_as_float(order_key(ex)));
                        }
                    }
                }
                __syncwarp();
                // rank each own band entry among the band entries of both sub-lists by
                // (canonical score desc, key asc); the first `need` are kept
                uint32_t obm[kMaskWords];
    #pragma unroll
                for (int w = 0; w < kMaskWords; ++w) obm[w] = __shfl_xor_sync(kFull, bm[w], 1);
                if (rescore) {
                    const uint32_t oth_s = smem_u32(frowbuf + (1 - fh) * Cfg::kCap);
    #pragma unroll
                    for (int w = 0; w < kMaskWords; ++w) {
                        for (uint32_t m = bm[w]; m != 0u; m &= m - 1u) {
                            const int qa = 32 * w + __ffs(m) - 1;
                            const uint2 ea = lds_u2(own_s + 8u * qa);
                            int rank = 0;
    #pragma unroll
                            for (int w2 = 0; w2 < kMaskWords; ++w2) {
                                for (uint32_t m2 = bm[w2]; m2 != 0u; m2 &= m2 - 1u) {
                                    const uint2 e = lds_u2(own_s + 8u * (32 * w2 + __ffs(m2) - 1));
                                    rank += (e.x > ea.x || (e.x == ea.x && e.y < ea.y)) ? 1 : 0;
                                }
                                for (uint32_t m2 = obm[w2]; m2 != 0u; m2 &= m2 - 1u) {
                                    const uint2 e = lds_u2(oth_s + 8u * (32 * w2 + __ffs(m2) - 1));
                                    rank += (e.x > ea.x || (e.x == ea.x && e.y < ea.y)) ? 1 : 0;
                                }
                            }
                            if (rank < need) sm[w] |= 1u << (qa & 31);
                        }
                    }
                }
                __syncwarp();  // the partner is done reading this sub-list before it is compacted

                // 3. compact kept keys in place, then merge the two lists
                int nsel = 0;
                if (work) {
                    uint32_t wa = own_s + 4u;  // .y of the next kept slot
    #pragma unroll
                    for (int ch = 0; ch < Cfg::kCap / 8; ++ch) {
                        if (ch < nch) {
                            // scores re-read from the list, a chunk at a time (x[] is not kept
                            // live across the band work); loads before the chunk's stores
                            uint2 e8[8];
    #pragma unroll
                            for (int u = 0; u < 8; ++u) e8[u] = lds_u2(own_s + 8u * (8 * ch + u));
    #pragma unroll
                            for (int u = 0; u < 8; ++u) {
                                const int q = 8 * ch + u;
                                // band entries (rescored in place) by their selection bit,
                                // the others by their approximate score: above U (certain),
                                // or at least W when the whole band is kept
                                const float sq = q < nown ? __uint_as_float(e8[u].x) : -INFINITY;
                                const bool inbm = (bm[q >> 5] >> (q & 31)) & 1u;
                                const bool keep = inbm ? ((sm[q >> 5] >> (q & 31)) & 1u) != 0u : (sq > U || sq >= W);
                                sts_u32_if(wa, e8[u].y, keep);
                                wa += keep ? 8u : 0u;
                            }
                        }
                    }
                    nsel = (int)((wa - own_s - 4u) >> 3);
                }
                const int nsel_oth = __shfl_xor_sync(kFull, nsel, 1);
                __syncwarp();
                const int nA = fh ? nsel_oth : nsel;
                const int nB = fh ? nsel : nsel_oth;
                const int ntot = nA + nB;
                const int mfront = (ntot + 1) >> 1;
                const int mcount = fh ? ntot - mfront : mfront;
                const int steps = (int)__reduce_max_sync(kFull, work ? (unsigned)mcount : 0u);
                // The merged rows are staged in the (now idle) k' tile ring, 256 B per row
                // with the 16-byte groups XOR-swizzled by row, then written out with
                // coalesced 16-byte stores.
                const uint32_t stage_s = smem_u32(sB);
                {
                    const uint32_t LA = smem_u32(frowbuf) + 4u;             // .y fields
                    const uint32_t LB = LA + 8u * Cfg::kCap;
                    // Lane 2r merges from the front (smaller key first), lane 2r+1 from the
                    // back (larger key first).  Keys are compared as u = j (front) or
                    // u = 0x7fffffff - j (back) unsigned, so one compare serves both lanes
                    // and an exhausted list (j = -1) sorts last.  Each list keeps its
                    // current and next key in registers; the shared-memory read that
                    // refills the taken list's next key is issued a step before it is
                    // compared, and no step branches.
                    const int dir = fh ? -1 : 1;
                    const uint32_t ubase = fh ? 0x7fffffffu : 0u;
                    auto key_u = [&](uint32_t base, int idx, int n) -> uint32_t {
                        const uint32_t j = lds_u32_or(base + 8u * (uint32_t)idx, work && idx >= 0 && idx < n, 0xffffffffu);
                        return fh ? ubase - j : j;  // j = -1 maps to 0x80000000 (back) or 0xffffffff (front)
                    };
                    int ia = fh ? nA - 1 : 0, ib = fh ? nB - 1 : 0;
                    uint32_t ua = key_u(LA, ia, nA), ua2 = key_u(LA, ia + dir, nA);
                    uint32_t ub = key_u(LB, ib, nB), ub2 = key_u(LB, ib + dir, nB);
                    const uint32_t srow = stage_s + 256u * frow;
                    const int swz = (frow & 7) << 2;
                    const int col0 = fh ? ntot - 1 : 0;
                    for (int st = 0; st < steps; ++st) {
                        const bool ta = ua < ub;
                        const uint32_t u = ta ? ua : ub;
                        const int col = col0 + dir * st;
                        sts_u32_if(srow + 4u * (uint32_t)(col ^ swz), fh ? ubase - u : u, work && st < mcount);
                        // the taken list advances: its next key becomes current, and the key
                        // after that is read
                        const int nidx = (ta ? ia : ib) + 2 * dir;
                        const uint32_t fetched = key_u(ta ? LA : LB, nidx, ta ? nA : nB);
                        ia += ta ? dir : 0;
                        ib += ta ? 0 : dir;
                        ua = ta ? ua2 : ua;
                        ub = ta ? ub : ub2;
                        ua2 = ta ? fetched : ua2;
                        ub2 = ta ? ub2 : fetched;
                    }
                    if (work && fh) {
                        for (int q = ntot; q < K; ++q) sts_f32(srow + 4u * (uint32_t)(q ^ swz), __int_as_float(-1));
                    }
                }
                __syncwarp();
                {
                    // this warp's 16 rows: r0 + 16 * hf + rin, finished by lane pair rin
                    const unsigned workmask = __ballot_sync(kFull, work);
                    const int rbase = r0 + 16 * hf;
                    if ((K & 3) == 0) {
                        const int per_row = K >> 2;
                        // f / per_row by a reciprocal: (f + 0.5) / per_row stays at least
                        // 1/32 away from an integer for f < 256, per_row <= 16
                        const float inv_pr = 1.f / (float)per_row;
                        for (int f = lane; f < 16 * per_row; f += 32) {
                            const int rin = (int)(((float)f + 0.5f) * inv_pr), v = f - rin * per_row;
                            if ((workmask >> (2 * rin)) & 1u) {
                                const int rrow = rbase + rin;
                                const uint4 val = lds_u4(stage_s + 256u * rrow + 16u * (uint32_t)(v ^ (rrow & 7)));
                                const size_t oid = (size_t)bh * Nq + (size_t)(i0 + rrow);
                                *(reinterpret_cast<uint4*>(p.out + oid * K) + v) = val;
                            }
                        }
                    } else {
                        for (int f = lane; f < 16 * K; f += 32) {
                            const int rin = f / K, c = f - rin * K;
                            if ((workmask >> (2 * rin)) & 1u) {
                                const int rrow = rbase + rin;
                                const uint32_t val = lds_u32(stage_s + 256u * rrow + 4u * (uint32_t)(c ^ ((rrow & 7) << 2)));
                                const size_t oid = (size_t)bh * Nq + (size_t)(i0 + rrow);
                                p.out[oid * K + c] = (int32_t)val;
                            }
                        }
                    }
                }
                if (to_fallback && fh == 0) {
                    const int pos = atomicAdd(p.fb_count, 1);
                    p.fb_list[pos] = (int32_t)orow_id;
                }
            }
            // the bulk copies of Wq land before the CTA retires
            if (p.q_in != nullptr && ew == 0 && lane == 0 && !mbar_wait(wtbar, 0u)) atomicOr(p.status, 16);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// --------------------------------------------------- exact fallback for listed rows

// Streaming exact selection by one warp (the same rule as the exact CTA selector):
// items arrive 32 at a time in ascending key order; an item is admitted when its
// order key beats theta, the K-th best kept so far, and the buffer wb (32 EPL
// entries) is cut back to the K best whenever it could overflow.  Ties keep the
// earlier slot, that is the lower key index.
template <int EPL>
__device__ __forceinline__ void stream_chunk(bool valid, uint32_t key, uint32_t j, int K, uint2* wb, int& cnt,
                                             uint32_t& theta, int lane, unsigned lt) {
    constexpr int CAP = 32 * EPL;
    const bool adm = valid && key > theta;
    const unsigned bal = __ballot_sync(kFull, adm);
    if (adm) wb[cnt + __popc(bal & lt)] = make_uint2(key, j);
    cnt += __popc(bal);
    __syncwarp();
    if (cnt > CAP - 32) {
        uint32_t u[EPL], jv[EPL];
        bool val[EPL], keep[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            const int q = lane + 32 * e;
            val[e] = q < cnt;
            const uint2 t = val[e] ? wb[q] : make_uint2(0u, 0u);
            u[e] = t.x;
            jv[e] = t.y;
        }
        uint32_t Tk;
        warp_topk_mask<EPL>(u, val, K, keep, &Tk);
        __syncwarp();
        int outpos = 0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            const unsigned kb = __ballot_sync(kFull, keep[e]);
            if (keep[e]) wb[outpos + __popc(kb & lt)] = make_uint2(u[e], jv[e]);
            outpos += __popc(kb);
        }
        __syncwarp();
        cnt = outpos;
        theta = Tk;
    }
}

// The K best of the warp's buffer in slot order (ascending key index): emit(pos,
// entry) for each; returns how many.
template <int EPL, typename Emit>
__device__ __forceinline__ int stream_finish(int cnt, int K, const uint2* wb, int lane, unsigned lt, Emit&& emit) {
    uint32_t u[EPL], jv[EPL];
    bool val[EPL], keep[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const int q = lane + 32 * e;
        val[e] = q < cnt;
        const uint2 t = val[e] ? wb[q] : make_uint2(0u, 0u);
        u[e] = t.x;
        jv[e] = t.y;
    }
    if (cnt > K) {
        warp_topk_mask<EPL>(u, val, K, keep);
    } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) keep[e] = val[e];
    }
    int outpos = 0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const unsigned kb = __ballot_sync(kFull, keep[e]);
        if (keep[e]) emit(outpos + __popc(kb & lt), make_uint2(u[e], jv[e]));
        outpos += __popc(kb);
    }
    return outpos;
}

// Position, key range and rows of listed row `row` (global query-row index).
struct FbRow {
    const float* qrow;
    const float* kbase;
    int i, n;
};
template <int kD>
__device__ __forceinline__ FbRow fb_row(const float* qp, const float* kp, long long row, int H, int Hkv, int N,
                                        int Nq, int q0, int causal) {
    const long long bh = row / Nq;
    const int i = q0 + (int)(row - bh * Nq);  // position in the key sequence
    const int b = (int)(bh / H);
    const int h = (int)(bh - (long long)b * H);
    const int g = h / (H / Hkv);
    return FbRow{qp + row * kD, kp + (size_t)(b * Hkv + g) * N * kD, i, causal ? min(i + 1, N) : N};
}

// One warp per listed row: canonical scores on CUDA cores, streaming selection.
template <int EPL, int kD = kR, bool kBias = true>
__global__ void __launch_bounds__(256)
exact_rows_kernel(const float* __restrict__ qp, const float* __restrict__ kp, const float* __restrict__ bias,
                  int L, int H, int Hkv, int N, int Nq, int q0, int K, float scale, int causal,
                  const int* __restrict__ fb_count,
                  const int32_t* __restrict__ fb_list, int32_t* __restrict__ out) {
    constexpr int CAP = 32 * EPL;
    __shared__ uint2 sbuf[8][CAP];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned lt = lanemask_lt();
    const int total = *reinterpret_cast<const volatile int*>(fb_count);
    uint2* wb = sbuf[warp];
    for (int idx = blockIdx.x * 8 + warp; idx < total; idx += gridDim.x * 8) {
        const long long row = fb_list[idx];
        const FbRow r = fb_row<kD>(qp, kp, row, H, Hkv, N, Nq, q0, causal);
        uint32_t theta = 0u;
        int cnt = 0;
        for (int j0 = 0; j0 < r.n; j0 += 32) {
            const int j = j0 + lane;
            const bool valid = j < r.n;
            uint32_t key = 0u;
            if (valid) key = order_key(canonical_score<kD, kBias>(r.qrow, r.kbase + (size_t)j * kD, bias, L, r.i, j, scale));
            stream_chunk<EPL>(valid, key, (uint32_t)j, K, wb, cnt, theta, lane, lt);
        }
        int32_t* orow = out + row * K;
        const int nout = stream_finish<EPL>(cnt, K, wb, lane, lt, [&](int pos, uint2 e) { orow[pos] = (int32_t)e.y; });
        for (int q = nout + lane; q < K; q += 32) orow[q] = -1;
        __syncwarp();
    }
}

// Long rows: one CTA per listed row.  Each of its 8 warps streams one eighth of the
// row's keys (in key order) to its own K best, and warp 0 streams the 8 lists, in
// segment order, to the row's K best.  The K best of the row are among the union of
// the segments' K best, and that stream is still in ascending key order, so the
// result is the single-warp one.
template <int EPL, int kD = kR, bool kBias = true>
__global__ void __launch_bounds__(256)
exact_rows_split_kernel(const float* __restrict__ qp, const float* __restrict__ kp, const float* __restrict__ bias,
                        int L, int H, int Hkv, int N, int Nq, int q0, int K, float scale, int causal,
                        const int* __restrict__ fb_count, const int32_t* __restrict__ fb_list,
                        int32_t* __restrict__ out) {
    constexpr int CAP = 32 * EPL;
    __shared__ uint2 sbuf[8][CAP];
    __shared__ uint2 sres[8][CAP];
    __shared__ int scnt[8];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned lt = lanemask_lt();
    const int total = *reinterpret_cast<const volatile int*>(fb_count);
    uint2* wb = sbuf[warp];
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
        const long long row = fb_list[idx];
        const FbRow r = fb_row<kD>(qp, kp, row, H, Hkv, N, Nq, q0, causal);
        const int seg = ((r.n + 8 * 32 - 1) / (8 * 32)) * 32;  // a multiple of 32 keys per warp
        const int s0 = min(r.n, warp * seg), s1 = min(r.n, s0 + seg);
        uint32_t theta = 0u;
        int cnt = 0;
        for (int j0 = s0; j0 < s1; j0 += 32) {
            const int j = j0 + lane;
            const bool valid = j < s1;
            uint32_t key = 0u;
            if (valid) key = order_key(canonical_score<kD, kBias>(r.qrow, r.kbase + (size_t)j * kD, bias, L, r.i, j, scale));
            stream_chunk<EPL>(valid, key, (uint32_t)j, K, wb, cnt, theta, lane, lt);
        }
        uint2* res = sres[warp];
        const int nres = stream_finish<EPL>(cnt, K, wb, lane, lt, [&](int pos, uint2 e) { res[pos] = e; });
        if (lane == 0) scnt[warp] = nres;
        __syncthreads();
        if (warp == 0) {
            theta = 0u;
            cnt = 0;
            for (int w = 0; w < 8; ++w) {
                const int m = scnt[w];
                for (int p0 = 0; p0 < m; p0 += 32) {
                    const int p = p0 + lane;
                    const bool valid = p < m;
                    const uint2 e = valid ? sres[w][p] : make_uint2(0u, 0u);
                    stream_chunk<EPL>(valid, e.x, e.y, K, wb, cnt, theta, lane, lt);
                }
            }
            int32_t* orow = out + row * K;
            const int nout = stream_finish<EPL>(cnt, K, wb, lane, lt, [&](int pos, uint2 e) { orow[pos] = (int32_t)e.y; });
            for (int q = nout + lane; q < K; q += 32) orow[q] = -1;
        }
        __syncthreads();  // sres and scnt are reused by the next row
    }
}

// ------------------------------------------------------ per-row final choice

struct FinalParams {
    const uint2* lists;
    const int* counts;
    const float2* rowinfo;
    const float* bias;
    const float* qp32;
    const float* kp32;
    const __nv_bfloat16* q_in;  // as in TcParams
    const float* wt;
    int32_t* out;
    int* fb_count;
    int32_t* fb_list;
    long long rows;
    int L, H, Hkv, N, K, Nq, q0, nqb;
    float scale;
};

// One warp per query row.  The row's two candidate sub-lists A and B (one per
// column half, keys ascending, at most kCap each) are loaded as entry
// q = lane + 32 e of A ++ B.  With more than K candidates, the K-th best
// approximate score x_K splits them: let top = the best score below x_K when
// exactly K entries reach x_K, else x_K itself, and m2 = 2 delta plus rounding
// slack.  Entries above U = top + m2 are certainly in the exact top K, entries
// below W = x_K - m2 certainly not; when the band [W, U] holds more entries than
// the free slots, its entries are rescored with the canonical fp32 formula and
// the best by (score desc, key asc) fill the slots.  The kept keys of A and B
// are then merged by rank into ascending order, -1 padded.  When the band holds
// more than kMaxBand entries, every candidate is rescored canonically and the
// exact top K is taken among them.  Rows whose lists overflowed or whose inputs
// are not finite go to the exact fallback list.
template <int kCap, int kMaxOut, int kD = kR, bool kBias = true>
__global__ void __launch_bounds__(256) final_select_kernel(const FinalParams p) {
    constexpr int kEPL = 2 * kCap / 32;  // candidate entries per lane
    static_assert(kEPL * 32 == 2 * kCap && kMaxBand <= 32, "list and band layout");
    __shared__ int skept[8][2][kMaxOut];
    __shared__ int sband[8][32];
    __shared__ __align__(16) float swt[128 * 64];  // on-demand q' rows: Wq transposed, [d][c]
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned lt = lanemask_lt();
    const int K = p.K;
    if (p.q_in != nullptr) {
        for (int e = threadIdx.x; e < 128 * 64 / 4; e += blockDim.x)
            reinterpret_cast<float4*>(swt)[e] = __ldg(reinterpret_cast<const float4*>(p.wt) + e);
        __syncthreads();
    }
    for (long long row = (long long)blockIdx.x * 8 + warp; row < p.rows; row += (long long)gridDim.x * 8) {
        const int ca = p.counts[2 * row], cb = p.counts[2 * row + 1];
        bool fallback = ca < 0 || cb < 0 || ca > kCap || cb > kCap;
        if (!fallback) {
            const long long bh = row / p.Nq;
            const int il = (int)(row - bh * p.Nq);
            const uint2* LA = p.lists + ((size_t)bh * p.nqb + il / kTileM) * (2 * kTileM * (size_t)kCap) +
                              (size_t)(2 * (il % kTileM)) * kCap;  // contiguous sub-lists (wide layout)
            const uint2* LB = LA + kCap;
            const int tot = ca + cb;
            float sv[kEPL];
            uint32_t jv[kEPL];
            bool val[kEPL], keep[kEPL];
#pragma unroll
            for (int e = 0; e < kEPL; ++e) {
                const int q = lane + 32 * e;
                val[e] = q < tot;
                uint2 t = make_uint2(0u, 0u);
                if (val[e]) t = q < ca ? LA[q] : LB[q - ca];
                sv[e] = __uint_as_float(t.x);
                jv[e] = t.y;
                keep[e] = val[e];
            }
            if (tot > K) {
                uint32_t u[kEPL];
#pragma unroll
                for (int e = 0; e < kEPL; ++e) u[e] = order_key(sv[e]);
                uint32_t T;
                int ties;
                warp_kth_key_search<kEPL>(u, val, K, T, ties);
                unsigned nge = 0;
                uint32_t below = 0u;  // order keys of finite scores are never 0
#pragma unroll
                for (int e = 0; e < kEPL; ++e) {
                    if (val[e]) {
                        if (u[e] >= T) ++nge;
                        else below = max(below, u[e]);
                    }
                }
                nge = __reduce_add_sync(kFull, nge);
                below = __reduce_max_sync(kFull, below);
                const float xk = key_to_float(T);
                const float top = ((int)nge == K && below != 0u) ? key_to_float(below) : xk;
                const float fdelta = p.rowinfo[row].y;
                const float sl = fmaxf(fabsf(top), fabsf(xk));
                const float m2 = 2.f * fdelta + (sl + 2.f * fdelta) * kTwoPowM22;
                const float U = top + m2, W = xk - m2;
                unsigned n_in = 0, nb = 0;
                bool band[kEPL];
#pragma unroll
                for (int e = 0; e < kEPL; ++e) {
                    band[e] = val[e] && sv[e] >= W && sv[e] <= U;
                    n_in += (val[e] && sv[e] > U) ? 1u : 0u;
                    nb += band[e] ? 1u : 0u;
                }
                n_in = __reduce_add_sync(kFull, n_in);
                nb = __reduce_add_sync(kFull, nb);
                const int need = K - (int)n_in;
                if ((int)nb == need) {
#pragma unroll
                    for (int e = 0; e < kEPL; ++e) keep[e] = val[e] && sv[e] >= W;
                } else if (nb > (unsigned)kMaxBand) {
                    // band wider than a lane each: rescore every candidate with the
                    // canonical formula and take the exact top K among them (the list
                    // holds every key that can be in it), ties to the lower key index
                    const long long bh = row / p.Nq;
                    const int ipos = p.q0 + (int)(row - bh * p.Nq);
                    const int b = (int)(bh / p.H);
                    const int g = (int)(bh - (long long)b * p.H) / (p.H / p.Hkv);
                    const float* qrow = p.qp32 + (size_t)row * kD;
                    const float* kbase = p.kp32 + (size_t)(b * p.Hkv + g) * p.N * kD;
                    if (p.q_in != nullptr) {
                        warp_canon_q2(p.q_in + row * 128, p.q_in + row * 128, swt, swt + 4096,
                                      const_cast<float*>(qrow), nullptr, lane);
                        __syncwarp();
                    }
                    uint32_t ek[kEPL];
#pragma unroll
                    for (int e = 0; e < kEPL; ++e)
                        ek[e] = val[e] ? order_key(canonical_score<kD, kBias, true>(
                                             qrow, kbase + (size_t)jv[e] * kD, p.bias, p.L, ipos, (int)jv[e], p.scale))
                                       : 0u;
                    uint32_t Te;
                    int ties;
                    warp_kth_key_search<kEPL>(ek, val, K, Te, ties);
                    // the K best are {ek > Te} plus the `ties` lowest keys with ek == Te
                    bool taken[kEPL];
#pragma unroll
                    for (int e = 0; e < kEPL; ++e) taken[e] = false;
                    for (int tsel = 0; tsel < ties; ++tsel) {
                        uint32_t jmin = 0xffffffffu;
#pragma unroll
                        for (int e = 0; e < kEPL; ++e)
                            if (val[e] && ek[e] == Te && !taken[e]) jmin = min(jmin, jv[e]);
                        jmin = __reduce_min_sync(kFull, jmin);
#pragma unroll
                        for (int e = 0; e < kEPL; ++e)
                            if (val[e] && ek[e] == Te && jv[e] == jmin) taken[e] = true;
                    }
#pragma unroll
                    for (int e = 0; e < kEPL; ++e) keep[e] = val[e] && (ek[e] > Te || taken[e]);
                } else {
                    // band entries to lanes 0..nb-1, in (e, lane) order
                    const long long bh = row / p.Nq;
                    const int ipos = p.q0 + (int)(row - bh * p.Nq);
                    const int b = (int)(bh / p.H);
                    const int g = (int)(bh - (long long)b * p.H) / (p.H / p.Hkv);
                    int slot[kEPL];
                    int base = 0;
#pragma unroll
                    for (int e = 0; e < kEPL; ++e) {
                        const unsigned bal = __ballot_sync(kFull, band[e]);
                        slot[e] = base + __popc(bal & lt);
                        if (band[e]) sband[warp][slot[e]] = (int)jv[e];
                        base += __popc(bal);
                    }
                    if (p.q_in != nullptr)
                        warp_canon_q2(p.q_in + row * 128, p.q_in + row * 128, swt, swt + 4096,
                                           const_cast<float*>(p.qp32) + row * kD, nullptr, lane);
                    __syncwarp();
                    uint32_t ek = 0u;
                    int jj = INT_MAX;
                    if (lane < (int)nb) {
                        jj = sband[warp][lane];
                        const float ex = canonical_score<kD, kBias, true>(
                            p.qp32 + (size_t)row * kD, p.kp32 + ((size_t)(b * p.Hkv + g) * p.N + jj) * kD, p.bias,
                            p.L, ipos, jj, p.scale);
                        ek = order_key(ex);
                    }
                    int rank = 0;
                    for (int l2 = 0; l2 < (int)nb; ++l2) {
                        const uint32_t e2 = __shfl_sync(kFull, ek, l2);
                        const int j2 = __shfl_sync(kFull, jj, l2);
                        rank += (e2 > ek || (e2 == ek && j2 < jj)) ? 1 : 0;
                    }
                    const unsigned sel = __ballot_sync(kFull, lane < (int)nb && rank < need);
#pragma unroll
                    for (int e = 0; e < kEPL; ++e)
                        keep[e] = val[e] && (sv[e] > U || (band[e] && ((sel >> slot[e]) & 1u)));
                    __syncwarp();  // sband is rewritten for the next row
                }
            }
            if (!fallback) {
                // kept keys of each list, compacted in list order (ascending keys)
                int* SA = skept[warp][0];
                int* SB = skept[warp][1];
                int na = 0, nbk = 0;
#pragma unroll
                for (int e = 0; e < kEPL; ++e) {
                    const bool isA = lane + 32 * e < ca;
                    const bool kA = keep[e] && isA, kB = keep[e] && !isA;
                    const unsigned balA = __ballot_sync(kFull, kA);
                    const unsigned balB = __ballot_sync(kFull, kB);
                    const int li = isA ? na + __popc(balA & lt) : nbk + __popc(balB & lt);
                    if (kA && li < kMaxOut) SA[li] = (int)jv[e];
                    if (kB && li < kMaxOut) SB[li] = (int)jv[e];
                    na += __popc(balA);
                    nbk += __popc(balB);
                }
                na = min(na, kMaxOut);
                nbk = min(nbk, kMaxOut);
                __syncwarp();
                // merge path: lane l writes output positions 4l .. 4l+3 (kMaxOut <= 128);
                // the split of position 4l between the two ascending lists by binary
                // search, then four merge steps
                const int n = na + nbk;
                const int p0 = 4 * lane;
                int outv[4] = {-1, -1, -1, -1};
                if (p0 < n) {
                    int lo = max(0, p0 - nbk), hi = min(p0, na);
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (SA[mid] < SB[p0 - 1 - mid]) lo = mid + 1; else hi = mid;
                    }
                    int ia = lo, ib = p0 - lo;
#pragma unroll
                    for (int s2 = 0; s2 < 4; ++s2) {
                        if (p0 + s2 < n) {
                            const bool takeA = ib >= nbk || (ia < na && SA[ia] < SB[ib]);
                            outv[s2] = takeA ? SA[ia] : SB[ib];
                            ia += takeA ? 1 : 0;
                            ib += takeA ? 0 : 1;
                        }
                    }
                }
                int32_t* orow = p.out + row * K;
                if ((K & 3) == 0) {
                    if (p0 < K) *reinterpret_cast<int4*>(orow + p0) = make_int4(outv[0], outv[1], outv[2], outv[3]);
                } else {
#pragma unroll
                    for (int s2 = 0; s2 < 4; ++s2)
                        if (p0 + s2 < K) orow[p0 + s2] = outv[s2];
                }
                __syncwarp();  // skept is rewritten for the next row
            }
        }
        if (fallback && p.q_in != nullptr)
            warp_canon_q2(p.q_in + row * 128, p.q_in + row * 128, swt, swt + 4096,
                               const_cast<float*>(p.qp32) + row * kD, nullptr, lane);
        if (fallback && lane == 0) {
            const int pos = atomicAdd(p.fb_count, 1);
            p.fb_list[pos] = (int32_t)row;
        }
    }
}


// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// (rows x cols) fp16 row-major matrix -> 128-row x 64-column boxes with the
// 128-byte swizzle (a row of cols > 64 takes cols / 64 boxes).
bool make_row_map(CUtensorMap* map, const void* base, unsigned long long rows, int cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)kTileM};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t record(cudaError_t e) {
    if (e == cudaSuccess) note_launch();
    return e;
}

// Workspace of one tensor-core selection over row length kD: fp16 copies of the
// query and key rows, per-row multipliers and bounds, key and bias statistics,
// the fallback list, the window images and (lists in global memory) the
// candidate sub-lists of every row slot of every query block with their lengths.
size_t tc_workspace_bytes(int B, int H, int Hkv, int Nq, int N, int K, int kD) {
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t rq = (size_t)B * H * Nq, rk = (size_t)B * Hkv * N;
    const int nqb = (Nq + kTileM - 1) / kTileM, tiles_n = (N + kTileN - 1) / kTileN;
    size_t total = al(rq * kD * 2) + al(rk * kD * 2) + al(rq * sizeof(float2)) +
                   al((kStatWords * (size_t)B * Hkv + 2) * 4) + al(rq * 4) +
                   (nqb > 0 && tiles_n > 0 ? al((size_t)window_count(nqb, tiles_n) * kWinBytes) +
                                                  al((size_t)window_count(nqb, tiles_n) * 2 * kTileM * 4)
                                            : 0) +
                   al(rq * 4) + al(64 * 128 * 4);
    const bool wide = K > kNarrowMaxK;
    if (wide || kD > 64) {
        const size_t lrows = (size_t)B * H * nqb * kTileM;
        const int cap = wide ? TcCfg<true>::kCap : (kD > 64 ? TcCfg<false, 128>::kCap : TcCfg<false, 64>::kCap);
        total += al(lrows * 2 * (size_t)cap * sizeof(uint2)) + al(rq * 2 * sizeof(int));
    }
    return total;
}

// The exact selector for the rows listed in fb_list (their count is on the device):
// a warp per row, or for long rows (N >= kSplitRowsMinN) a CTA per row.
constexpr int kSplitRowsMinN = 8192;
template <int EPL, int kD, bool kBias>
cudaError_t launch_exact_rows(const RouterTcArgs& a, int Nq, const int* counters, const int32_t* fb_list,
                              cudaStream_t stream) {
    const int nsm = device_sm_count();
    if (a.N >= kSplitRowsMinN)
        exact_rows_split_kernel<EPL, kD, kBias><<<nsm, 256, 0, stream>>>(a.qp32, a.kp32, a.bias, a.L, a.H, a.Hkv,
                                                                          a.N, Nq, a.q0, a.K, a.scale, a.causal,
                                                                          counters, fb_list, a.out);
    else
        exact_rows_kernel<EPL, kD, kBias><<<2 * nsm, 256, 0, stream>>>(a.qp32, a.kp32, a.bias, a.L, a.H, a.Hkv, a.N,
                                                                        Nq, a.q0, a.K, a.scale, a.causal, counters,
                                                                        fb_list, a.out);
    return record(cudaGetLastError());
}

// One selection: prep kernels, the tensor-core kernel, then (lists in global
// memory) the warp-per-row final choice, then the exact fallback rows.
// kBias: router scores (pos_bias added); without it the oracle's scaled dot
// products.
template <int kD, bool kBias>
cudaError_t launch_tc(const RouterTcArgs& a, cudaStream_t stream) {
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    const int Nq = a.Nq > 0 ? a.Nq : a.N;
    const size_t rq = (size_t)a.B * a.H * Nq, rk = (size_t)a.B * a.Hkv * a.N;
    char* w = static_cast<char*>(a.ws);
    __half* q16 = reinterpret_cast<__half*>(w);
    w += al(rq * kD * 2);
    __half* k16 = reinterpret_cast<__half*>(w);
    w += al(rk * kD * 2);
    float2* rowinfo = reinterpret_cast<float2*>(w);
    w += al(rq * sizeof(float2));
    uint32_t* stats = reinterpret_cast<uint32_t*>(w);
    uint32_t* gstats = stats + kStatWords * (size_t)a.B * a.Hkv;
    w += al((kStatWords * (size_t)a.B * a.Hkv + 2) * 4);
    int32_t* fb_list = reinterpret_cast<int32_t*>(w);
    w += al(rq * 4);
    const int nqb = (Nq + kTileM - 1) / kTileM, tiles_n = (a.N + kTileN - 1) / kTileN;
    const int ndiag = window_count(nqb, tiles_n);
    float* wtab = reinterpret_cast<float*>(w);
    w += al((size_t)ndiag * kWinBytes);
    float* wmax = reinterpret_cast<float*>(w);
    w += al((size_t)ndiag * 2 * kTileM * 4);
    float* rowub = reinterpret_cast<float*>(w);
    w += al(rq * 4);
    float* wt = reinterpret_cast<float*>(w);  // Wq transposed (on-demand canonical q' rows)
    w += al(64 * 128 * 4);
    const bool wide = a.K > kNarrowMaxK;
    const bool global_lists = wide || kD > 64;
    const int cap = wide ? TcCfg<true, kD>::kCap : TcCfg<false, kD>::kCap;
    uint2* lists = nullptr;
    int* counts = nullptr;
    if (global_lists) {
        lists = reinterpret_cast<uint2*>(w);
        w += al((size_t)a.B * a.H * nqb * kTileM * 2 * (size_t)cap * sizeof(uint2));
        counts = reinterpret_cast<int*>(w);
    }
    int* counters = a.counters;  // [0] fallback rows, [1] status

    cudaError_t e = cudaMemsetAsync(stats, 0, (kStatWords * (size_t)a.B * a.Hkv + 2) * 4, stream);
    if (e != cudaSuccess) return e;

    const int BG = a.B * a.Hkv;
    {
        dim3 grid((a.N + 255) / 256, BG);
        kstats_kernel<kD><<<grid, 256, 0, stream>>>(a.kp32, a.N, stats);
        if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
        if (kBias) {
            bias_stats_kernel<<<8, 256, 0, stream>>>(a.bias, 2 * a.L, gstats);
            if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
        }
        dim3 g2((unsigned)(((long long)a.N * (kD / 4) + 255) / 256), BG);
        kconvert_kernel<kD><<<g2, 256, 0, stream>>>(a.kp32, k16, a.N, stats);
        if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
        if (a.qproj != nullptr) {
            const QPrepArgs qa{a.qproj->x, a.qproj->w, wt, (long long)rq, q16, rowinfo, rowub, stats, gstats,
                               counters + 1, a.H, a.Hkv, Nq, a.scale};
            if ((e = launch_qproj_tc(qa, stream)) != cudaSuccess) return e;
        } else {
            qprep_kernel<kD><<<(unsigned)((rq * 8 + 255) / 256), 256, 0, stream>>>(
                a.qp32, q16, rowinfo, rowub, (long long)rq, a.H, a.Hkv, Nq, a.scale, stats, gstats);
            if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
        }
        // offset of bias-line index 0: the window of tile (qb, key tile) starts at
        // i - j + L = q0 + kTileN * (qb - key tile) + 127 + L (its first column
        // against its last row)
        const long long o_max = (long long)a.q0 + (long long)kTileN * (nqb - 1) + (kTileN - 1) + a.L;
        const long long nb = (long long)ndiag * 4 * kWinCopy;
        window_table_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, stream>>>(kBias ? a.bias : nullptr, a.L,
                                                                             a.causal, o_max, ndiag, wtab);
        if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
        if (tiles_n >= kSkipMinTiles) {  // read only by the build with the half-tile skip
            const long long nm = (long long)ndiag * 2 * kTileM;
            window_max_kernel<<<(unsigned)((nm + 255) / 256), 256, 0, stream>>>(wtab, ndiag, wmax);
            if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
        }
    }
    CUtensorMap tmA, tmB;
    if (!make_row_map(&tmA, q16, rq, kD) || !make_row_map(&tmB, k16, rk, kD)) return cudaErrorInvalidValue;
    const int smem_bytes = (int)(wide ? TcCfg<true, kD>::kSmemBytes : TcCfg<false, kD>::kSmemBytes);
    // the build with the half-tile skip when some query block reaches kSkipMinTiles key tiles
    const bool skip = tiles_n >= kSkipMinTiles;
    auto kern = wide ? (skip ? router_tc_kernel<true, kD, true> : router_tc_kernel<true, kD, false>)
                     : (skip ? router_tc_kernel<false, kD, true> : router_tc_kernel<false, kD, false>);
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    TcParams prm;
    prm.rowinfo = rowinfo;
    prm.bias = a.bias;
    prm.qp32 = a.qp32;
    prm.q_in = a.qproj ? static_cast<const __nv_bfloat16*>(a.qproj->x) : nullptr;
    prm.wt = a.qproj ? wt : nullptr;
    prm.kp32 = a.kp32;
    prm.out = a.out;
    prm.fb_count = counters;
    prm.fb_list = fb_list;
    prm.status = counters + 1;
    prm.lists = lists;
    prm.counts = counts;
    prm.wtab = wtab;
    prm.wmax = wmax;
    prm.rowub = rowub;
    prm.L = a.L;
    prm.H = a.H;
    prm.Hkv = a.Hkv;
    prm.N = a.N;
    prm.K = a.K;
    prm.causal = a.causal;
    prm.Nq = Nq;
    prm.q0 = a.q0;
    prm.nqb = nqb;
    prm.scale = a.scale;
    const long long nblk = (long long)nqb * a.B * a.H;
    const int nsm = device_sm_count();
    if (!global_lists) {
        kern<<<(unsigned)nblk, kThreads, smem_bytes, stream>>>(tmA, tmB, prm);
        if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
        // rows sent to the exact selector (K + 32 candidates per warp: 4 entries per lane)
        return launch_exact_rows<4, kD, kBias>(a, Nq, counters, fb_list, stream);
    }
    kern<<<(unsigned)nblk, kThreads, smem_bytes, stream>>>(tmA, tmB, prm);
    if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
    FinalParams fp;
    fp.lists = lists;
    fp.counts = counts;
    fp.rowinfo = rowinfo;
    fp.bias = a.bias;
    fp.qp32 = a.qp32;
    fp.q_in = prm.q_in;
    fp.wt = prm.wt;
    fp.kp32 = a.kp32;
    fp.out = a.out;
    fp.fb_count = counters;
    fp.fb_list = fb_list;
    fp.rows = (long long)rq;
    fp.L = a.L;
    fp.H = a.H;
    fp.Hkv = a.Hkv;
    fp.N = a.N;
    fp.K = a.K;
    fp.Nq = Nq;
    fp.q0 = a.q0;
    fp.nqb = nqb;
    fp.scale = a.scale;
    const unsigned fblk = (unsigned)std::min<long long>(((long long)rq + 7) / 8, 8LL * nsm);
    if (wide) final_select_kernel<TcCfg<true, kD>::kCap, kWideMaxK, kD, kBias><<<fblk, 256, 0, stream>>>(fp);
    else final_select_kernel<TcCfg<false, kD>::kCap, kNarrowMaxK, kD, kBias><<<fblk, 256, 0, stream>>>(fp);
    if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
    // rows sent to the exact selector (K + 32 candidates per warp: 6 entries per lane for K <= 160)
    if (wide) return launch_exact_rows<6, kD, kBias>(a, Nq, counters, fb_list, stream);
    return launch_exact_rows<4, kD, kBias>(a, Nq, counters, fb_list, stream);
}

// bf16 rows -> fp32 rows (the oracle's canonical scores read fp32), 8 values per thread.
__global__ void widen_bf16_kernel(const __nv_bfloat16* __restrict__ in, float* __restrict__ out, long long n8) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n8) return;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(in) + t);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        f[2 * u] = __uint_as_float(w[u] << 16);
        f[2 * u + 1] = __uint_as_float(w[u] & 0xffff0000u);
    }
    float4* o = reinterpret_cast<float4*>(out) + 2 * t;
    o[0] = make_float4(f[0], f[1], f[2], f[3]);
    o[1] = make_float4(f[4], f[5], f[6], f[7]);
}

}  // namespace

bool make_row_map_16(CUtensorMap* map, const void* base, bool bf16, unsigned long long rows, int cols,
                     int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
              const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool router_tc_supported(int r, int K) { return r == kR && K >= 1 && K <= kWideMaxK; }

size_t router_tc_workspace_bytes(int B, int H, int Hkv, int Nq, int N, int K) {
    return tc_workspace_bytes(B, H, Hkv, Nq, N, K, kR);
}

cudaError_t launch_router_tc(const RouterTcArgs& a, cudaStream_t stream) {
    if (a.qproj != nullptr && (a.qproj->out != a.qp32 || a.qproj->R != kR || !qproj_tc_supported(*a.qproj)))
        return cudaErrorInvalidValue;
    return launch_tc<kR, true>(a, stream);
}

bool oracle_tc_supported(int D, int K) { return D == kOracleD && K >= 1 && K <= kWideMaxK; }

size_t oracle_tc_workspace_bytes(int B, int H, int Hkv, int N, int K, int dtype) {
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t rq = (size_t)B * H * N, rk = (size_t)B * Hkv * N;
    size_t total = al(tc_workspace_bytes(B, H, Hkv, N, N, K, kOracleD));
    if (dtype != kF32) total += al(rq * kOracleD * 4) + al(rk * kOracleD * 4);
    return total;
}

cudaError_t launch_oracle_tc(const OracleTcArgs& o, cudaStream_t stream) {
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t rq = (size_t)o.B * o.H * o.N, rk = (size_t)o.B * o.Hkv * o.N;
    char* w = static_cast<char*>(o.ws);
    const float* q32 = static_cast<const float*>(o.q);
    const float* k32 = static_cast<const float*>(o.k);
    char* tcws = w;
    w += al(tc_workspace_bytes(o.B, o.H, o.Hkv, o.N, o.N, o.K, kOracleD));
    if (o.dtype != kF32) {
        float* qw = reinterpret_cast<float*>(w);
        w += al(rq * kOracleD * 4);
        float* kw = reinterpret_cast<float*>(w);
        const long long nq8 = (long long)(rq * kOracleD / 8), nk8 = (long long)(rk * kOracleD / 8);
        widen_bf16_kernel<<<(unsigned)((nq8 + 255) / 256), 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(o.q), qw, nq8);
        cudaError_t e = record(cudaGetLastError());
        if (e != cudaSuccess) return e;
        widen_bf16_kernel<<<(unsigned)((nk8 + 255) / 256), 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(o.k), kw, nk8);
        if ((e = record(cudaGetLastError())) != cudaSuccess) return e;
        q32 = qw;
        k32 = kw;
    }
    RouterTcArgs a{q32, k32, nullptr, 1, o.B, o.H, o.Hkv, o.N, o.K, o.causal, o.scale, o.out, tcws, o.counters};
    return launch_tc<kOracleD, false>(a, stream);
}

}  // namespace ossa
