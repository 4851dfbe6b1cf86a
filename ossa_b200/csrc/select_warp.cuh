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

// keep[e] = the entry is among the K largest (see warp_kth_key's tie rule).
template <int EPL>
__device__ __forceinline__ void warp_topk_mask(const uint32_t (&u)[EPL], const bool (&val)[EPL], int K,
                                               bool (&keep)[EPL], uint32_t* T_out = nullptr) {
    uint32_t T;
    int ties;
    warp_kth_key<EPL>(u, val, K, T, ties);
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
