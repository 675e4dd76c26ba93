// Device-side communicator descriptor and the cross-GPU block barrier used by
// every peer-memory collective.
//
// Every rank owns one "symmetric heap": a device allocation of identical size
// and layout on each GPU, mapped into every other rank's address space (CUDA
// IPC across processes, peer access within one process). A kernel addresses
// rank p's copy of heap offset `off` as `peer_base[p] + off`.
//
// Heap layout (offsets in bytes):
//   [0, kFlagBytes)               signal pad: u64 flags[kMaxBlocks][kMaxRanks]
//   [stage_off, +2*slot_bytes)    staging slots A and B
//   [user_off, heap_bytes)        user symmetric tensors (bump allocated)
//
// Barrier protocol: block b of rank r stores `epoch` into
// flags[b][r] on every peer p (st.release.sys), then waits until its own
// flags[b][p] >= epoch for all p (ld.acquire.sys). Epochs come from a device
// resident call counter, so a CUDA graph replay gets fresh epochs, and they
// grow monotonically for the lifetime of the communicator. Every wait is
// bounded by `timeout_ns` of %globaltimer; on expiry the block records the
// failure in the host-mapped status word and the kernel exits normally.
#pragma once
#include "common.cuh"

namespace nexar {

NEXAR_D unsigned long long* flag_ptr(const CommDev& c, int owner, int block, int src) {
  return reinterpret_cast<unsigned long long*>(c.peer_base[owner]) + block * kMaxRanks + src;
}

NEXAR_D void record_timeout(const CommDev& c, int peer, int op, unsigned long long epoch) {
  volatile DeviceStatus* s = c.status;
  s->rank = (unsigned)peer;
  s->op = (unsigned)op;
  s->block = blockIdx.x;
  s->epoch = epoch;
  __threadfence_system();
  s->code = kStatusWaitTimeout;
  __threadfence_system();
}

NEXAR_D void record_check(const CommDev& c, int op, unsigned int id, unsigned long long value,
                          unsigned long long limit) {
  volatile DeviceStatus* s = c.status;
  s->rank = (unsigned)value;
  s->op = (unsigned)op;
  s->block = id;
  s->epoch = limit;
  __threadfence_system();
  s->code = kStatusCheckFailed;
  __threadfence_system();
}

// Entry checks of a collective kernel (when c.checks is set): every block
// evaluates the same launch arguments, so all blocks agree and return
// together before touching memory. `bytes` must not exceed `limit`.
NEXAR_D bool entry_ok(const CommDev& c, int op, int root = 0, unsigned long long bytes = 0,
                      unsigned long long limit = ~0ull) {
#ifndef NEXAR_NO_DEVICE_CHECKS
  if (!c.checks) return true;
  unsigned int id = 0;
  unsigned long long v = 0, lim = 0;
  if (c.world < 1 || c.world > kMaxRanks || c.rank < 0 || c.rank >= c.world) {
    id = kCheckComm;
    v = (unsigned long long)c.rank;
    lim = (unsigned long long)c.world;
  } else if (root < 0 || root >= c.world) {
    id = kCheckRoot;
    v = (unsigned long long)(long long)root;
    lim = (unsigned long long)c.world;
  } else if (bytes > limit) {
    id = kCheckBytes;
    v = bytes;
    lim = limit;
  }
  if (id != 0) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_check(c, op, id, v, lim);
    return false;
  }
#endif
  return true;
}

// Block-wide barrier with every peer's block of the same index. Returns false
// (uniformly across the block) if any wait timed out (or, with device checks
// on, if the epoch is not above the one this block stored last time).
NEXAR_D bool block_barrier(const CommDev& c, unsigned long long epoch, int op) {
  __syncthreads();
  int ok = 1;
  const int p = threadIdx.x;
#ifndef NEXAR_NO_DEVICE_CHECKS
  if (c.checks) {
    __shared__ int s_epoch_ok;
    if (threadIdx.x == 0) {
      const unsigned long long prev = ld_acquire_sys(flag_ptr(c, c.rank, blockIdx.x, c.rank));
      s_epoch_ok = prev < epoch;
      if (!s_epoch_ok) record_check(c, op, kCheckEpoch, prev, epoch);
    }
    __syncthreads();
    if (!s_epoch_ok) return false;
  }
#endif
  if (p < c.world) {
    fence_sys();
    st_release_sys(flag_ptr(c, p, blockIdx.x, c.rank), epoch);
    const unsigned long long* mine = flag_ptr(c, c.rank, blockIdx.x, p);
    if (ld_acquire_sys(mine) < epoch) {
      const unsigned long long t0 = globaltimer_ns();
      unsigned int spins = 0;
      while (ld_acquire_sys(mine) < epoch) {
        if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > c.timeout_ns) {
          record_timeout(c, p, op, epoch);
          ok = 0;
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// Per-kernel bookkeeping: read the call index at entry; the last block to
// finish advances it. Consecutive kernels of one communicator are stream
// ordered, so every block of the next kernel observes the new value.
NEXAR_D unsigned long long call_index(const CommDev& c) {
  return *reinterpret_cast<volatile unsigned long long*>(c.ctrl);
}
NEXAR_D void finish_call(const CommDev& c, unsigned long long call) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int prev = atomicAdd(reinterpret_cast<unsigned int*>(c.ctrl + 1), 1u);
    if (prev == gridDim.x - 1) {
      reinterpret_cast<volatile unsigned int*>(c.ctrl + 1)[0] = 0u;
      reinterpret_cast<volatile unsigned long long*>(c.ctrl)[0] = call + 1;
      __threadfence();
    }
  }
}
NEXAR_D unsigned long long epoch_of(unsigned long long call, int phase) {
  return call * 4ull + (unsigned long long)phase + 1ull;
}

// Contiguous block-partition of `total` units, each block range a multiple
// of `align` units (the last one may be shorter).
NEXAR_HD void block_range(unsigned long long total, unsigned int nblocks, unsigned int b,
                          unsigned long long align, unsigned long long* lo,
                          unsigned long long* hi) {
  unsigned long long per = (total + nblocks - 1) / nblocks;
  per = (per + align - 1) / align * align;
  unsigned long long l = per * b;
  if (l > total) l = total;
  unsigned long long h = l + per;
  if (h > total) h = total;
  *lo = l;
  *hi = h;
}

}  // namespace nexar
