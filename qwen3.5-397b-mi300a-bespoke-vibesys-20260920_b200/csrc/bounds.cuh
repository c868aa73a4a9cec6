// Debug bounds checks and scratch canaries (compiled in with -DQB_BOUNDS; the release build
// compiles every check to `true` and allocates no canary).
//
// Index checks: a kernel that indexes memory with a value it read from memory (a token id, a
// paged-KV row, an expert id, a lane) checks it against the capacity the host passed. A value
// out of range records, in the device status word, ERR_BOUNDS, the check's site, the value and
// the capacity (first failure wins), and the kernel skips that access. Nothing traps: the host
// reads the word as it reads every other device error (utils/devstatus.py), so the failing site
// is named without faulting the GPU.
//
// Canaries: in the debug build every scratch buffer the bindings allocate gets 256 bytes of
// 0xA5 after its end; after the kernel that used it, a one-block check kernel compares them and
// records ERR_CANARY with the buffer's site if any byte changed (a write past the end).
//
// The status word is reached through a file-scope device pointer per translation unit, set once
// per device by that unit's install function (bindings.cpp, when the word is created).
#pragma once
#include "common.cuh"
#include "kernels.h"  // BoundsSite, CANARY_BYTES, CANARY_BYTE

namespace qb {

#ifdef QB_BOUNDS
static __device__ int* qb_bounds_word = nullptr;

__device__ __forceinline__ void bounds_record(int code, int site, long v, long hi) {
  int* w = qb_bounds_word;
  if (w != nullptr && atomicCAS(w, 0, code) == 0) {
    w[1] = site;
    w[2] = (int)v;
    w[3] = (int)hi;
  }
}

__device__ __forceinline__ bool bounds_ok(int site, long v, long hi) {
  if (v >= 0 && v < hi) return true;
  bounds_record(ERR_BOUNDS, site, v, hi);
  return false;
}

#define QB_BOUNDS_INSTALL(fn) \
  int fn(int* word) { return (int)cudaMemcpyToSymbol(qb_bounds_word, &word, sizeof(word)); }
#else
__device__ __forceinline__ bool bounds_ok(int, long, long) { return true; }
#define QB_BOUNDS_INSTALL(fn) \
  int fn(int*) { return 0; }
#endif

}  // namespace qb
