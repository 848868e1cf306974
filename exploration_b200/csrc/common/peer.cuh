// System-scope flag accesses and the wall clock used by the peer-memory
// kernels (symmetric heap barrier, gradient reduction). Peer memory is
// another GPU's allocation mapped through CUDA IPC; the owner's L2 is the
// point of coherence, so a release store after a system fence publishes
// everything this GPU wrote before it.
#pragma once

#include <cstdint>

#include "util.cuh"

namespace eb {

EB_DEVICE void store_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

EB_DEVICE void store_relaxed_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

EB_DEVICE unsigned int load_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

EB_DEVICE uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

}  // namespace eb
