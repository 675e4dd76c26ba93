// Mixture-of-experts expert parallelism over NVLink peer memory (sm_100a).
//
// One expert per GPU (E == world). A forward pass is
//   route    (local)   top-2 of the router logits per token, softmax over the
//                      two chosen logits, per-expert slot counts and each
//                      slot's position within its expert bucket;
//   counts   (device all-gather of the [E] count vector, W*E ints);
//   dispatch (fused)   all-to-all with the token permutation fused in: every
//                      token row is stored straight into row
//                      (prefix of earlier sources + local position) of the
//                      expert GPU's symmetric receive buffer; the last block
//                      to finish publishes "dispatch done" to every peer and
//                      waits for theirs, so the expert GEMMs that follow on the
//                      stream see every row;
//   experts  (tcgen05 GEMMs on the received rows);
//   combine  (fused)   after an "expert outputs ready" handshake, every
//                      token pulls its two expert output rows from the expert
//                      GPUs (plain peer loads), scales them by the gates and
//                      sums them in fp32 (top-1 then top-2, so results are
//                      deterministic).
// The reference has only a plain all_to_all (nexar/src/collective/alltoall.rs);
// the fusion with routing permutation and gating is new. All waits are
// bounded and record the silent rank in the status word.
#include "coll.cuh"
#include "coll_api.h"
#include "moe_api.h"

namespace nexar {

namespace {
constexpr int kMoeThreads = 256;

NEXAR_D unsigned long long* moe_flag(const CommDev& c, int owner, size_t off, int src) {
  return reinterpret_cast<unsigned long long*>(c.peer_base[owner] + off) + src;
}

NEXAR_D bool wait_ge(const unsigned long long* p, unsigned long long target, unsigned long long timeout_ns) {
  if (ld_acquire_sys(p) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  unsigned int spins = 0;
  while (ld_acquire_sys(p) < target) {
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > timeout_ns) return false;
  }
  return true;
}

// One warp per token.
template <typename TL>
__global__ void __launch_bounds__(kMoeThreads) k_moe_route(const TL* __restrict__ logits, int T, int E,
                                                           int* __restrict__ slot_expert, int* __restrict__ slot_pos,
                                                           float* __restrict__ slot_gate, int* __restrict__ counts) {
  const int warp = (blockIdx.x * kMoeThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const TL* row = logits + (size_t)warp * E;
  float best = -INFINITY, second = -INFINITY;
  int ib = -1, is = -1;
  for (int e = lane; e < E; e += 32) {
    const float v = (float)row[e];
    if (v > best || (v == best && (ib < 0 || e < ib))) {
      second = best;
      is = ib;
      best = v;
      ib = e;
    } else if (v > second || (v == second && (is < 0 || e < is))) {
      second = v;
      is = e;
    }
  }
  // warp merge of (best, second) pairs; ties go to the lower expert id
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float b2 = __shfl_xor_sync(0xffffffffu, best, o), s2 = __shfl_xor_sync(0xffffffffu, second, o);
    const int ib2 = __shfl_xor_sync(0xffffffffu, ib, o), is2 = __shfl_xor_sync(0xffffffffu, is, o);
    float c[4] = {best, second, b2, s2};
    int ci[4] = {ib, is, ib2, is2};
    float nb = -INFINITY, ns = -INFINITY;
    int nib = -1, nis = -1;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (ci[k] < 0 || ci[k] == nib || ci[k] == nis) continue;
      if (c[k] > nb || (c[k] == nb && ci[k] < nib)) {
        ns = nb;
        nis = nib;
        nb = c[k];
        nib = ci[k];
      } else if (c[k] > ns || (c[k] == ns && ci[k] < nis)) {
        ns = c[k];
        nis = ci[k];
      }
    }
    best = nb;
    second = ns;
    ib = nib;
    is = nis;
  }
  if (lane == 0) {
    // softmax over the two selected logits
    const float g2 = 1.f / (1.f + __expf(best - second));
    const float g1 = 1.f - g2;
    slot_expert[2 * warp] = ib;
    slot_expert[2 * warp + 1] = is;
    slot_gate[2 * warp] = g1;
    slot_gate[2 * warp + 1] = g2;
    slot_pos[2 * warp] = atomicAdd(&counts[ib], 1);
    slot_pos[2 * warp + 1] = atomicAdd(&counts[is], 1);
  }
}

// One warp per slot: copy the token row into the expert GPU's receive buffer.
__global__ void __launch_bounds__(kMoeThreads) k_moe_dispatch(CommDev c, const __nv_bfloat16* __restrict__ x, int T,
                                                              int d, const int* __restrict__ slot_expert,
                                                              int* __restrict__ slot_pos,
                                                              const int* __restrict__ counts_all,
                                                              unsigned long long recv_off, int capacity,
                                                              unsigned int* ticket) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpMoeDispatch)) {
    finish_call(c, call);
    return;
  }
  const unsigned long long epoch = epoch_of(call, 0);
  __shared__ int base[kMaxRanks];
  const int E = c.world;
  if (threadIdx.x < E) {
    // rows of earlier sources come first in expert e's buffer
    int b = 0;
    for (int s = 0; s < c.rank; ++s) b += counts_all[s * E + threadIdx.x];
    base[threadIdx.x] = b;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (kMoeThreads / 32);
  const int packs = d / 8;
  for (int slot = (blockIdx.x * kMoeThreads + threadIdx.x) >> 5; slot < 2 * T; slot += warps) {
    const int e = slot_expert[slot];
    const int pos = base[e] + slot_pos[slot];
    if (lane == 0) slot_pos[slot] = pos < capacity ? pos : -1;  // global row (or dropped)
    if (pos >= capacity) continue;
    const __nv_bfloat16* src = x + (size_t)(slot >> 1) * d;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(c.peer_base[e] + recv_off) + (size_t)pos * d;
    int i = lane;
    for (; i + 96 < packs; i += 128) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = ld16(src + (i + 32 * u) * 8);
#pragma unroll
      for (int u = 0; u < 4; ++u) st16(dst + (i + 32 * u) * 8, v[u]);
    }
    for (; i < packs; i += 32) st16(dst + i * 8, ld16(src + i * 8));
  }
  // The last block publishes "dispatch done" to every peer and waits for theirs.
  __syncthreads();
  __shared__ unsigned int t;
  if (threadIdx.x == 0) {
    __threadfence_system();
    t = atomicAdd(ticket, 1u);
  }
  __syncthreads();
  if (t == gridDim.x - 1) {
    if (threadIdx.x == 0) {
      *ticket = 0u;
      fence_sys();
    }
    __syncthreads();
    if ((int)threadIdx.x < c.world) {
      const int p = threadIdx.x;
      st_release_sys(moe_flag(c, p, kMoeDispatchDoneOff, c.rank), epoch);
      if (!wait_ge(moe_flag(c, c.rank, kMoeDispatchDoneOff, p), epoch, c.timeout_ns))
        record_timeout(c, p, kOpMoeDispatch, epoch);
    }
  }
  finish_call(c, call);
}

// Backward of combine (one warp per slot): slot (t, k) stores scale[slot] *
// g[t] into global row slot_pos[slot] of expert slot_expert[slot]'s buffer
// (rows already placed by the forward dispatch; -1 = dropped, skipped), then
// the same "dispatch done" handshake as k_moe_dispatch.
__global__ void __launch_bounds__(kMoeThreads) k_moe_dispatch_rows(CommDev c, const __nv_bfloat16* __restrict__ g,
                                                                   int T, int d, const int* __restrict__ slot_expert,
                                                                   const int* __restrict__ slot_pos,
                                                                   const float* __restrict__ slot_scale,
                                                                   unsigned long long dst_off, int capacity,
                                                                   unsigned int* ticket) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpMoeDispatch)) {
    finish_call(c, call);
    return;
  }
  const unsigned long long epoch = epoch_of(call, 0);
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (kMoeThreads / 32);
  const int packs = d / 8;
  for (int slot = (blockIdx.x * kMoeThreads + threadIdx.x) >> 5; slot < 2 * T; slot += warps) {
    const int e = slot_expert[slot];
    const int pos = slot_pos[slot];
    if (pos < 0 || pos >= capacity || e < 0 || e >= c.world) continue;
    const float sc = slot_scale ? slot_scale[slot] : 1.f;
    const __nv_bfloat16* src = g + (size_t)(slot >> 1) * d;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(c.peer_base[e] + dst_off) + (size_t)pos * d;
    for (int i = lane; i < packs; i += 32) {
      const uint4 a = ld16(src + i * 8);
      const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
      uint4 r;
      __nv_bfloat162* hr = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(ha[k]);
        hr[k] = __floats2bfloat162_rn(sc * f.x, sc * f.y);
      }
      st16(dst + i * 8, r);
    }
  }
  __syncthreads();
  __shared__ unsigned int t;
  if (threadIdx.x == 0) {
    __threadfence_system();
    t = atomicAdd(ticket, 1u);
  }
  __syncthreads();
  if (t == gridDim.x - 1) {
    if (threadIdx.x == 0) {
      *ticket = 0u;
      fence_sys();
    }
    __syncthreads();
    if ((int)threadIdx.x < c.world) {
      const int p = threadIdx.x;
      st_release_sys(moe_flag(c, p, kMoeDispatchDoneOff, c.rank), epoch);
      if (!wait_ge(moe_flag(c, c.rank, kMoeDispatchDoneOff, p), epoch, c.timeout_ns))
        record_timeout(c, p, kOpMoeDispatch, epoch);
    }
  }
  finish_call(c, call);
}

// One warp per token: out[t] = g1 * E_{e1}[pos1] + g2 * E_{e2}[pos2].
__global__ void __launch_bounds__(kMoeThreads) k_moe_combine(CommDev c, __nv_bfloat16* __restrict__ out, int T, int d,
                                                             const int* __restrict__ slot_expert,
                                                             const int* __restrict__ slot_pos,
                                                             const float* __restrict__ slot_gate,
                                                             unsigned long long eout_off) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpMoeCombine)) {
    finish_call(c, call);
    return;
  }
  const unsigned long long epoch = epoch_of(call, 0);
  // Handshake: every rank's expert outputs are complete before anyone reads.
  int ok = 1;
  if ((int)threadIdx.x < c.world) {
    const int p = threadIdx.x;
    if (blockIdx.x == 0) {
      fence_sys();
      st_release_sys(moe_flag(c, p, kMoeExpertDoneOff, c.rank), epoch);
    }
    ok = wait_ge(moe_flag(c, c.rank, kMoeExpertDoneOff, p), epoch, c.timeout_ns);
    if (!ok) record_timeout(c, p, kOpMoeCombine, epoch);
  }
  if (__syncthreads_and(ok)) {
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kMoeThreads / 32);
    const int packs = d / 8;
    for (int tok = (blockIdx.x * kMoeThreads + threadIdx.x) >> 5; tok < T; tok += warps) {
      const int e1 = slot_expert[2 * tok], e2 = slot_expert[2 * tok + 1];
      const int p1 = slot_pos[2 * tok], p2 = slot_pos[2 * tok + 1];
      const float g1 = p1 >= 0 ? slot_gate[2 * tok] : 0.f, g2 = p2 >= 0 ? slot_gate[2 * tok + 1] : 0.f;
      const __nv_bfloat16* r1 = reinterpret_cast<const __nv_bfloat16*>(c.peer_base[e1] + eout_off) + (size_t)max(p1, 0) * d;
      const __nv_bfloat16* r2 = reinterpret_cast<const __nv_bfloat16*>(c.peer_base[e2] + eout_off) + (size_t)max(p2, 0) * d;
      __nv_bfloat16* o = out + (size_t)tok * d;
      for (int i = lane; i < packs; i += 32) {
        const uint4 a = p1 >= 0 ? ld16_volatile(r1 + i * 8) : make_uint4(0, 0, 0, 0);
        const uint4 b = p2 >= 0 ? ld16_volatile(r2 + i * 8) : make_uint4(0, 0, 0, 0);
        const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
        uint4 r;
        __nv_bfloat162* hr = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 fa = __bfloat1622float2(ha[k]), fb = __bfloat1622float2(hb[k]);
          hr[k] = __floats2bfloat162_rn(g1 * fa.x + g2 * fb.x, g1 * fa.y + g2 * fb.y);
        }
        st16(o + i * 8, r);
      }
    }
  }
  finish_call(c, call);
}
}  // namespace

cudaError_t moe_route(const void* logits, bool logits_bf16, int T, int E, int* slot_expert, int* slot_pos,
                      float* slot_gate, int* counts, cudaStream_t s) {
  if (E < 2 || E > 64) return cudaErrorInvalidValue;
  const int blocks = (T * 32 + kMoeThreads - 1) / kMoeThreads;
  if (logits_bf16)
    k_moe_route<__nv_bfloat16><<<blocks, kMoeThreads, 0, s>>>((const __nv_bfloat16*)logits, T, E, slot_expert, slot_pos, slot_gate, counts);
  else
    k_moe_route<float><<<blocks, kMoeThreads, 0, s>>>((const float*)logits, T, E, slot_expert, slot_pos, slot_gate, counts);
  return cudaGetLastError();
}

cudaError_t moe_dispatch(const CommDev& c, const __nv_bfloat16* x, int T, int d, const int* slot_expert,
                         int* slot_pos, const int* counts_all, unsigned long long recv_off, int capacity,
                         unsigned int* ticket, cudaStream_t s) {
  if (d % 8) return cudaErrorInvalidValue;
  int blocks = (2 * T * 32 + kMoeThreads - 1) / kMoeThreads;
  if (blocks > 148 * 4) blocks = 148 * 4;
  k_moe_dispatch<<<blocks, kMoeThreads, 0, s>>>(c, x, T, d, slot_expert, slot_pos, counts_all, recv_off, capacity,
                                                ticket);
  return cudaGetLastError();
}

cudaError_t moe_dispatch_rows(const CommDev& c, const __nv_bfloat16* g, int T, int d, const int* slot_expert,
                              const int* slot_pos, const float* slot_scale, unsigned long long dst_off, int capacity,
                              unsigned int* ticket, cudaStream_t s) {
  if (d % 8) return cudaErrorInvalidValue;
  int blocks = (2 * T * 32 + kMoeThreads - 1) / kMoeThreads;
  if (blocks > 148 * 4) blocks = 148 * 4;
  k_moe_dispatch_rows<<<blocks, kMoeThreads, 0, s>>>(c, g, T, d, slot_expert, slot_pos, slot_scale, dst_off, capacity,
                                                     ticket);
  return cudaGetLastError();
}

cudaError_t moe_combine(const CommDev& c, __nv_bfloat16* out, int T, int d, const int* slot_expert,
                        const int* slot_pos, const float* slot_gate, unsigned long long eout_off, cudaStream_t s) {
  if (d % 8) return cudaErrorInvalidValue;
  int blocks = (T * 32 + kMoeThreads - 1) / kMoeThreads;
  if (blocks > 148 * 4) blocks = 148 * 4;
  k_moe_combine<<<blocks, kMoeThreads, 0, s>>>(c, out, T, d, slot_expert, slot_pos, slot_gate, eout_off);
  return cudaGetLastError();
}

}  // namespace nexar
