// Host-visible descriptor of one phase of a peer exchange over NVLink
// (symmetric memory): a producer kernel publishes "my data for this phase is
// complete" into every rank's signal array; consumer kernels wait until every
// rank has published the same epoch.
#pragma once
#include <stdint.h>

namespace dsv4 {

struct PeerSync {
  uint32_t* const* peer_sig;   // [world] device pointers to each rank's signal array (uint32 [phases * world])
  const uint32_t* sig;         // this rank's signal array (the waits read it)
  int* done;                   // this rank's CTA completion counter of the phase (zero at rest)
  uint32_t* epoch;             // this rank's epoch counter of the phase
  int phase, world, rank;
};

}  // namespace dsv4
