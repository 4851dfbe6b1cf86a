// Warp-cooperative selection primitives over a small candidate list held as
// EPL entries per lane (entry p = lane + 32 * e, list order = position order).
#pragma once

#include "common.cuh"

namespace ossa {

// Finds the K-th largest of the valid 32-bit order keys (K >= 1 and at least K
// valid entries).  On return T is that key and `ties` the number of entries
// equal to T that belong to the K largest when ties are broken by position
// (earliest first): the K largest are exactly {u > T} plus the first `ties`
// entries with u == T.  Radix select from the highest bit where the keys
// differ, stopping early once every entry of the current prefix group is taken.
template <int EPL>
__device__ __forceinline__ void warp_kth_key(const uint32_t (&u)[EPL], const bool (&val)[EPL], int K,
                                             uint32_t& T, int& ties) {
    uint32_t mx = 0u, mn = 0xffffffffu;
    unsigned nvalid = 0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        if (val[e]) {
            mx = max(mx, u[e]);
            mn = min(mn, u[e]);
            ++nvalid;
        }
    }
    mx = __reduce_max_sync(kFull, mx);
    mn = __reduce_min_sync(kFull, mn);
    int count = (int)__reduce_add_sync(kFull, nvalid);
    int kk = K;
    if (mx == mn) {
        T = mx;
        ties = kk;
        return;
    }
    const int hb = 31 - __clz(mx ^ mn);
    uint32_t mask = ~((2u << hb) - 1u);
    uint32_t prefix = mx & mask;
#pragma unroll 1
    for (int bit = hb; bit >= 0; --bit) {
        const uint32_t bm = 1u << bit;
        const uint32_t m2 = mask | bm;
        const uint32_t cand = prefix | bm;
        unsigned c = 0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) c += (val[e] && (u[e] & m2) == cand) ? 1u : 0u;
        c = __reduce_add_sync(kFull, c);
        if ((int)c >= kk) {
            prefix = cand;
            count = (int)c;
        } else {
            kk -= (int)c;
            count -= (int)c;
        }
        mask = m2;
        if (count == kk) {
            // every entry of the prefix group is among the K largest
            uint32_t lo = 0xffffffffu;
#pragma unroll
            for (int e = 0; e < EPL; ++e)
                if (val[e] && (u[e] & mask) == prefix) lo = min(lo, u[e]);
            T = __reduce_min_sync(kFull, lo);
            unsigned nt = 0;
#pragma unroll
            for (int e = 0; e < EPL; ++e) nt += (val[e] && u[e] == T) ? 1u : 0u;
            ties = (int)__reduce_add_sync(kFull, nt);
            return;
        }
    }
    T = prefix;
    ties = kk;
}

// The same result as warp_kth_key (T = the K-th largest valid key, `ties` = how
// many entries equal to T belong to the K largest), found by searching the key
// range instead of walking its bits.  The bracket [lo, hi) keeps
// count(u >= lo) >= K > count(u >= hi); probes alternate between linear
// interpolation of that count (a few probes on spread-out scores) and bisection
// (at most 32 more probes on any input).  The search ends when count(u >= lo) is
// exactly K, so the K largest are {u >= lo} and T is their minimum, or when the
// bracket is one key wide, so T = lo.  Requires more than K valid entries.
template <int EPL>
__device__ __forceinline__ void warp_kth_key_search(const uint32_t (&u)[EPL], const bool (&val)[EPL], int K,
                                                    uint32_t& T, int& ties) {
    uint32_t mx = 0u, mn = 0xffffffffu;
    unsigned nvalid = 0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        if (val[e]) {
            mx = max(mx, u[e]);
            mn = min(mn, u[e]);
            ++nvalid;
        }
    }
    mx = __reduce_max_sync(kFull, mx);
    mn = __reduce_min_sync(kFull, mn);
    int clo = (int)__reduce_add_sync(kFull, nvalid);
    uint64_t lo = mn, hi = (uint64_t)mx + 1u;  // count(u >= hi) = 0
    int chi = 0;
#pragma unroll 1
    for (int it = 0; clo != K && hi - lo > 1u && it < 80; ++it) {
        uint64_t pr;
        if (it & 1) {
            pr = lo + ((hi - lo) >> 1);
        } else {
            const float f = ((float)(clo - K) + 0.5f) / (float)(clo - chi);
            pr = lo + (uint64_t)((double)f * (double)(hi - lo));
            pr = pr <= lo ? lo + 1u : (pr >= hi ? hi - 1u : pr);
        }
        const uint32_t p32 = (uint32_t)pr;
        unsigned c = 0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) c += (val[e] && u[e] >= p32) ? 1u : 0u;
        const int cc = (int)__reduce_add_sync(kFull, c);
        if (cc >= K) {
            lo = pr;
            clo = cc;
        } else {
            hi = pr;
            chi = cc;
        }
    }
    const uint32_t lo32 = (uint32_t)lo;
    uint32_t t = 0xffffffffu;
#pragma unroll
    for (int e = 0; e < EPL; ++e)
        if (val[e] && u[e] >= lo32) t = min(t, u[e]);
    T = __reduce_min_sync(kFull, t);
    unsigned gt = 0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) gt += (val[e] && u[e] > T) ? 1u : 0u;
    ties = K - (int)__reduce_add_sync(kFull, gt);
}

// keep[e] = the entry is among the K largest (see warp_kth_key's tie rule).
// Requires more than K valid entries (every caller compacts a list only then).
template <int EPL>
__device__ __forceinline__ void warp_topk_mask(const uint32_t (&u)[EPL], const bool (&val)[EPL], int K,
                                               bool (&keep)[EPL], uint32_t* T_out = nullptr) {
    uint32_t T;
    int ties;
    warp_kth_key_search<EPL>(u, val, K, T, ties);
    const unsigned lt = lanemask_lt();
    int seen = 0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const bool tie = val[e] && u[e] == T;
        const unsigned tb = __ballot_sync(kFull, tie);
        keep[e] = val[e] && (u[e] > T || (tie && seen + __popc(tb & lt) < ties));
        seen += __popc(tb);
    }
    if (T_out) *T_out = T;
}

}  // namespace ossa
