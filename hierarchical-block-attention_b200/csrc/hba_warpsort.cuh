// Warp-wide sorting of (score, id) pairs under the library's order -- score
// descending, then id ascending (hba_common.cuh `beats`): a 32-lane bitonic
// sort and a merge that keeps the best 32 of a sorted list and a sorted batch.
#pragma once

#include "hba_common.cuh"

namespace hba {

// Warp-wide (score, id) compare-exchange with the lane `stride` away under
// the library order (score desc, id asc); keep_better selects which of the
// pair this lane keeps.
HBA_DEVICE void cmpx(float& s, int& i, int stride, bool keep_better) {
  const float os = __shfl_xor_sync(0xffffffffu, s, stride);
  const int oi = __shfl_xor_sync(0xffffffffu, i, stride);
  if (keep_better ? beats(os, oi, s, i) : beats(s, i, os, oi)) {
    s = os;
    i = oi;
  }
}
// Bitonic sort of the warp's 32 (score, id) pairs, best in lane 0.
HBA_DEVICE void warp_sort32(float& s, int& i) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1)
      cmpx(s, i, stride, ((lane & stride) == 0) == ((lane & size) == 0));
}
// (ls, li) sorted best first <- best 32 of itself and the sorted batch (bs, bi).
HBA_DEVICE void warp_merge32(float& ls, int& li, float bs, int bi) {
  const int lane = threadIdx.x & 31;
  const float rs = __shfl_sync(0xffffffffu, bs, 31 - lane);
  const int ri = __shfl_sync(0xffffffffu, bi, 31 - lane);
  if (beats(rs, ri, ls, li)) {  // best 32 of the union, as a bitonic sequence
    ls = rs;
    li = ri;
  }
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) cmpx(ls, li, stride, (lane & stride) == 0);
}

// Offers one batch -- one (score, id) per lane, (-inf, INT_MAX) for none -- to
// the running list (ls, li): the best 32 seen so far, sorted best first.
// Only candidates that beat entry k-1 can change the top k: none -> nothing
// to do; an empty list takes the sorted batch; a few are inserted one by
// one; many are sorted and merged.  Warp-uniform control flow.
HBA_DEVICE void warp_offer(float& ls, int& li, float cs, int ci, int k) {
  const int lane = threadIdx.x & 31;
  const float ts = __shfl_sync(0xffffffffu, ls, k - 1);
  const int ti = __shfl_sync(0xffffffffu, li, k - 1);
  const bool cand = beats(cs, ci, ts, ti);
  const unsigned mask = __ballot_sync(0xffffffffu, cand);
  if (mask == 0u) return;
  if (__shfl_sync(0xffffffffu, li, 0) == 0x7fffffff) {  // empty list: the sorted batch
    warp_sort32(cs, ci);
    ls = cs;
    li = ci;
  } else if (__popc(mask) > 6) {
    if (!cand) {
      cs = neg_inf();
      ci = 0x7fffffff;
    }
    warp_sort32(cs, ci);
    warp_merge32(ls, li, cs, ci);
  } else {
    for (unsigned mm = mask; mm; mm &= mm - 1) {
      const int src = __ffs(mm) - 1;
      const float xs = __shfl_sync(0xffffffffu, cs, src);
      const int xi = __shfl_sync(0xffffffffu, ci, src);
      const int at = __popc(__ballot_sync(0xffffffffu, !beats(xs, xi, ls, li)));  // entries ahead of it
      const float ps = __shfl_up_sync(0xffffffffu, ls, 1);
      const int pi = __shfl_up_sync(0xffffffffu, li, 1);
      if (lane == at) {
        ls = xs;
        li = xi;
      } else if (lane > at) {
        ls = ps;
        li = pi;
      }
    }
  }
}

}  // namespace hba
