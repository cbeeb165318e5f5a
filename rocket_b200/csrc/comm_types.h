// Host/device shared types of the fused-collective layer (no device code).
#pragma once
#include <stdint.h>

namespace rkt {

constexpr int kMaxRanks = 8;

// Flag block layout (per rank, in its symmetric buffer): uint32 flags[kSites][kMaxRanks].
constexpr int kSites = 16;

struct PeerPtrs {
  uint8_t* base[kMaxRanks];   // every rank's symmetric buffer base (this rank's own included)
  int rank, world;
  uint64_t flag_off;          // byte offset of the flag block inside each buffer
  uint32_t* counters;         // this rank's local counters [3*kSites] (see layout below)
};

}  // namespace rkt
