// Device code shared by the MoE decode kernels (q4nx_moe.cu): the group
// table built from ascending-ID slot lists.
#pragma once

#include "moe_internal.cuh"
#include "rc_device.cuh"

namespace rc {

// ------------------------------------------------------------ grouping --
// One warp.  Reads the slot lists of T tokens (shared memory, or global data
// written by this CTA before a barrier), builds the ascending-ID group table.
// Scratch smem_mask / smem_gidx hold E+1 entries.
__device__ __forceinline__ void build_groups(const int32_t *slot_expert, int T, int k, int n_experts, MoeOwned own,
                             const MoeScratch &s, uint32_t *smem_mask, int *smem_gidx, int lane) {
  const int ne = n_experts + 1;
  for (int e = lane; e < ne; e += 32) smem_mask[e] = 0u;
  __syncwarp();
  for (int pr = lane; pr < T * k; pr += 32) {
    const int t = pr / k, r = pr - t * k;
    const int e = slot_expert[t * (k + 1) + r];
    if (e >= own.lo && e < own.hi) atomicOr(smem_mask + e, 1u << t);
    else if (e < 0 || e >= n_experts) atomicCAS(s.err, 0, kErrBadExpert);   // caller id out of range
  }
  __syncwarp();
  if (lane == 0) smem_mask[n_experts] = own.shared_mask;
  __syncwarp();
  int base = 0;
  for (int c = 0; c < ne; c += 32) {
    const int e = c + lane;
    const uint32_t m = e < ne ? smem_mask[e] : 0u;
    const uint32_t b = __ballot_sync(0xffffffffu, m != 0u);
    if (m) {
      const int gi = base + __popc(b & ((1u << lane) - 1u));
      s.group_expert[gi] = e;
      s.group_mask[gi] = m;
      smem_gidx[e] = gi;
    }
    base += __popc(b);
  }
  if (lane == 0) *s.n_groups = base;
  __syncwarp();
  for (int pr = lane; pr < T * (k + 1); pr += 32) {
    const int t = pr / (k + 1), r = pr - t * (k + 1);
    const int e = slot_expert[pr];
    bool mine;
    if (r < k) {
      mine = e >= own.lo && e < own.hi;
    } else {
      mine = e >= 0 && ((own.shared_mask >> t) & 1u);
    }
    if (mine) s.group_dst[smem_gidx[e] * kMoeMaxTokens + t] = pr;
  }
}

}  // namespace rc
