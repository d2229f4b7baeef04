// Device primitives shared by the peer-memory kernels (NVLink 5 / NVSwitch, sm_100a).
//
// * Time budgets are measured on the global nanosecond timer (%globaltimer), so
//   a budget means the same wall time at any SM clock (the power-capped clock
//   of a dense step is 1.3-1.5 GHz, the boost clock 1.97 GHz).
// * Every peer-memory kernel receives a device status block `st` (int32[4],
//   owned by the host, one per device):
//       st[0]  sticky error code (kErrPeerTimeout, kErrBounds, ...), 0 = ok
//       st[1]  identifier of the wait that gave up first (see PeerWait)
//       st[2]  largest received row count seen (capacity check)
//   Once st[0] is set every later wait returns at once, so a missing peer
//   costs one budget per process, not one per barrier; the host reads the
//   block once per step and raises.
// * Cross-rank barrier: one thread per peer release-stores this rank's epoch
//   into the peer's flag array and acquire-waits until the peer's epoch in
//   ours reached the same value.  Epochs only grow, so a rank that arrives
//   late passes at once.
// * Grid barrier for persistent kernels whose CTAs are co-resident
//   (cooperative launch): arrival counter + generation word, bounded.
#pragma once

#include "common.cuh"

namespace pm {

enum PeerWait : int {
  kWaitBarrier = 1,      // p2p_barrier kernel
  kWaitGrid = 2,         // grid barrier inside a persistent kernel
  kWaitEpCounts = 3,     // dispatch: count exchange
  kWaitEpRows = 4,       // dispatch: rows stored
  kWaitEpCombine = 5,    // combine: partial sums stored
  kWaitEpScatter = 6,    // backward scatter: output gradients stored
  kWhereIndexCheck = 7,  // an index read from data was out of range (bounds-checked debug build)
  kWaitSpExchange = 8,   // Ulysses sequence-parallel exchange
};

PM_DEVICE unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

PM_DEVICE void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
PM_DEVICE unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
PM_DEVICE unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
PM_DEVICE int ld_volatile_i32(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

PM_DEVICE bool status_failed(const int* st) { return ld_volatile_i32(st) != 0; }

PM_DEVICE void status_fail(int* st, int code, int where) {
  if (atomicCAS(st, 0, code) == 0) atomicExch(st + 1, where);
}

// Index check of the bounds-checked debug build for the peer-memory kernels: a bad index
// sets kErrBounds in the sticky status block and the caller skips the access.
#ifdef PLACEMOE_DEBUG_BOUNDS
PM_DEVICE bool peer_index_ok(int* st, bool cond) {
  if (!cond) status_fail(st, kErrBounds, kWhereIndexCheck);
  return cond;
}
#define PM_PEER_INDEX_OK(st, cond) (::pm::peer_index_ok((st), (cond)))
#else
#define PM_PEER_INDEX_OK(st, cond) (true)
#endif

// Threads 0..world-1 of the calling CTA take part (the caller syncs the CTA around it).
// Returns false when the budget ran out or an earlier wait had already failed.
PM_DEVICE bool peer_barrier_threads(const long long* peers, long long flags_off, int my_rank, int world,
                                    unsigned epoch, long long budget_ns, int* st, int where) {
  const int r = threadIdx.x;
  bool ok = true;
  if (r < world) {
    __threadfence_system();
    unsigned* remote = reinterpret_cast<unsigned*>(peers[r] + flags_off) + my_rank;
    st_release_sys(remote, epoch);
    const unsigned* mine = reinterpret_cast<const unsigned*>(peers[my_rank] + flags_off) + r;
    const unsigned long long start = now_ns();
    int polls = 0;
    while ((int)(ld_acquire_sys(mine) - epoch) < 0) {
      if ((++polls & 255) == 0) {
        if (status_failed(st)) { ok = false; break; }
        if ((long long)(now_ns() - start) > budget_ns) {
          status_fail(st, kErrPeerTimeout, where);
          ok = false;
          break;
        }
      }
    }
  }
  return ok;
}

// Bounded grid barrier.  bar[0] = arrivals, bar[1] = generation; both start at 0 and the
// arrivals word returns to 0 after every barrier.  All CTAs of the grid must be co-resident.
PM_DEVICE bool grid_barrier(unsigned* bar, long long budget_ns, int* st) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned gen = ld_acquire_gpu(bar + 1);
    __threadfence();
    const unsigned nblocks = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(bar, 1u) == nblocks - 1) {
      atomicExch(bar, 0u);
      __threadfence();
      atomicAdd(bar + 1, 1u);
    } else {
      const unsigned long long start = now_ns();
      int polls = 0;
      while (ld_acquire_gpu(bar + 1) == gen) {
        if ((++polls & 63) == 0) {
          if (status_failed(st)) { ok = 0; break; }
          if ((long long)(now_ns() - start) > budget_ns) {
            status_fail(st, kErrPeerTimeout, kWaitGrid);
            ok = 0;
            break;
          }
        }
      }
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

}  // namespace pm
