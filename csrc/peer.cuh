// Peer-memory signalling helpers shared by the NVLink collective kernels (symm.cu, decode.cu).
//
// Flags are 64-bit monotonic counters in IPC-shared memory: writers publish with a release store
// (or reduction) at system scope, readers poll with acquire loads, and every wait is bounded: after
// kPeerWait cycles the waiter records kErrTimeoutPeer in the device error word and gives up.
#pragma once

#include <c10/util/Exception.h>

#include <vector>

#include "common.cuh"

namespace vlm {

constexpr int kMaxRanks = 8;
// ~9 s at 1.9 GHz: generous for rank skew, still finite.
constexpr long long kPeerWait = 1ll << 34;

struct PeerTable {
  unsigned long long p[kMaxRanks];
};

VLM_DEV void store_release_sys(unsigned long long* addr, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}
VLM_DEV void add_release_sys(unsigned long long* addr, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}
VLM_DEV unsigned long long load_acquire_sys(const unsigned long long* addr) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
  return v;
}

// Wait until sig[base + p] >= target for every peer p != rank.  Called by one thread.
VLM_DEV bool wait_peers_at(const unsigned long long* sig, int64_t base, int W, int rank, unsigned long long target,
                           int* err, long long budget = kPeerWait) {
  const long long t0 = clock64();
  for (int p = 0; p < W; ++p) {
    if (p == rank) continue;
    const unsigned long long* a = sig + base + p;
    while (load_acquire_sys(a) < target) {
      if (clock64() - t0 > budget) {
        atomicCAS(err, 0, kErrTimeoutPeer);
        return false;
      }
    }
  }
  return true;
}

// Host: table of per-rank addresses (each plus byte_off).
inline PeerTable make_peer_table(const std::vector<int64_t>& ptrs, int64_t byte_off = 0) {
  TORCH_CHECK(!ptrs.empty() && ptrs.size() <= static_cast<size_t>(kMaxRanks), "peer table: 1..", kMaxRanks, " ranks");
  PeerTable t{};
  for (size_t i = 0; i < ptrs.size(); ++i) t.p[i] = static_cast<unsigned long long>(ptrs[i] + byte_off);
  return t;
}

}  // namespace vlm
