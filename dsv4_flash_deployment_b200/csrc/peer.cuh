// Device side of PeerSync (peer.h): release/acquire at system scope, the
// last-CTA publish, and the bounded wait.
//
// Epochs advance once per publish on every rank (every rank runs the same
// sequence of phases), so a waiter compares its peers' signal words with its
// own epoch, which its own publish of the phase has already advanced (the
// publish precedes the wait in stream order).  No reset between CUDA-graph
// replays is needed.
#pragma once
#include "common.cuh"
#include "peer.h"

namespace dsv4 {

DSV4_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

DSV4_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Called by every thread of every CTA after the CTA's last global store of the
// phase; the last CTA to arrive advances the epoch and release-stores it into
// slot [phase * world + rank] of every rank's signal array.  The world stores
// are issued by as many threads at once (one NVLink round trip instead of one
// per peer): thread 0's system fence, taken after it observed every other CTA's
// arrival, is ordered before them by the barrier.
DSV4_DEV void peer_publish_grid(const PeerSync& s) {
  if (s.done == nullptr) return;
  __shared__ uint32_t s_pub_epoch;
  __shared__ int s_pub_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int n_cta = (int)(gridDim.x * gridDim.y * gridDim.z);
    const bool last = atomicAdd(s.done, 1) == n_cta - 1;
    if (last) {
      *s.done = 0;
      const uint32_t ep = *s.epoch + 1u;
      *s.epoch = ep;
      __threadfence_system();
      s_pub_epoch = ep;
    }
    s_pub_last = last;
  }
  __syncthreads();
  if (s_pub_last && (int)threadIdx.x < s.world)
    st_release_sys(s.peer_sig[threadIdx.x] + s.phase * s.world + s.rank, s_pub_epoch);
}

// Single-CTA form (the caller's stores of the phase precede it).
DSV4_DEV void peer_publish_cta(const PeerSync& s) {
  __shared__ uint32_t s_pub_epoch;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t ep = *s.epoch + 1u;
    *s.epoch = ep;
    __threadfence_system();
    s_pub_epoch = ep;
  }
  __syncthreads();
  if ((int)threadIdx.x < s.world) st_release_sys(s.peer_sig[threadIdx.x] + s.phase * s.world + s.rank, s_pub_epoch);
}

// Thread 0 waits until every rank has published this rank's current epoch of
// the phase (bounded: on expiry it records ERR_PEER_TIMEOUT and the CTA goes on,
// so the host sees the error word instead of a hung GPU); then the CTA syncs.
DSV4_DEV void peer_wait(const PeerSync& s, uint32_t* err, uint32_t kid) {
  if (threadIdx.x == 0) {
    const uint32_t want = *reinterpret_cast<volatile const uint32_t*>(s.epoch);
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < s.world; ++r) {
      const uint32_t* slot = s.sig + s.phase * s.world + r;
      while ((int)(ld_acquire_sys(slot) - want) < 0) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report_error(err, ERR_PEER_TIMEOUT, kid, (uint32_t)(s.phase * 16 + r));
          r = s.world;
          break;
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace dsv4
