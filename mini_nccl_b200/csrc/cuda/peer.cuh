// Peer-memory context shared by the collective kernels (comm.cu) and the
// GEMMs fused with a collective (gemm.cu).
//
// A PeerCtx is everything a kernel needs to talk to the other ranks of one
// device communicator during one call: every rank's staging region for this
// call (already offset to the call's parity half), every rank's signal pad,
// the call's epoch (signals carry epoch+k, so a stale signal from an earlier
// call never satisfies a wait), and where to report a timeout.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace mnb {

constexpr int kMaxRanks = 16;
constexpr int kMaxBlocks = 256;
constexpr int kSigSlots = kMaxBlocks * kMaxRanks;
// Signal-pad rows 0..kMaxCommBlocks-1 are per-CTA barrier slots of the
// collectives; the last two rows hold per-source-rank arrival counters that
// the fused GEMMs bump with one remote atomic per CTA (monotonic: the host
// passes the value that means "every CTA of that rank has arrived").  A
// counter lets one thread per CTA wait on W words instead of every thread
// polling a slot per CTA, which floods L2 and starves incoming NVLink writes.
constexpr int kCountRow = kMaxBlocks - 1;    // all-gather -> GEMM pushes
constexpr int kRsCountRow = kMaxBlocks - 2;  // GEMM -> reduce-scatter tiles
constexpr int kMaxCommBlocks = kMaxBlocks - 2;

struct PeerCtx {
  void* data[kMaxRanks];     // staging region of every rank (this call's half)
  uint32_t* sig[kMaxRanks];  // signal pad of every rank: [kMaxBlocks][kMaxRanks]
  int rank, world;
  uint32_t epoch;
  uint32_t seq;
  volatile int* status;  // host-mapped {code, peer, block, seq}
  unsigned long long timeout_ns;
};

MNB_DEVICE void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Record a timeout in the status block (first writer wins).
MNB_DEVICE void report_timeout(volatile int* status, int peer, int block, uint32_t seq) {
  if (status[0] == 0) {
    status[1] = peer;
    status[2] = block;
    status[3] = static_cast<int>(seq);
    __threadfence_system();
    status[0] = kErrPeerTimeout;
  }
}

// Wait until *slot >= value (wrap-safe).  Gives up when the deadline passes
// or when another thread already reported an error; returns false then.
MNB_DEVICE bool wait_signal(const uint32_t* slot, uint32_t value, volatile int* status, int peer, int block,
                            uint32_t seq, unsigned long long timeout_ns, uint64_t t0) {
  uint32_t spins = 0;
  while (static_cast<int32_t>(ld_acquire_sys(slot) - value) < 0) {
    if ((++spins & 255u) == 0) {
      if (status[0] != 0) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        report_timeout(status, peer, block, seq);
        return false;
      }
      __nanosleep(spins < 4096 ? 64 : 256);
    }
  }
  return true;
}

}  // namespace mnb
