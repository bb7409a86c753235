// Device-side building blocks shared by the SE12 kernels (sm_100a only).
//
// * SE12 format constants (16x256 tiles, 15-entry codebook, escape code 15,
//   16 escape slots per tile) -- the on-disk format of lws.pack
//   (src/lws/domain/se12/tile.py:19-24 in the reference).
// * Thin inline-PTX wrappers: mbarrier, TMA tensor loads, 1-D bulk copies,
//   L2 cache policies, bf16 mma.sync, programmatic dependent launch.
// * Bounded waits: every spin on an mbarrier gives up after a wall-clock
//   limit, records an error code in the device status word and lets the
//   caller drain and return, so a logic error can never hang a GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace se12 {

constexpr int kTileRows = 16;
constexpr int kTileCols = 256;
constexpr int kTileSize = kTileRows * kTileCols;  // 4096 weights
constexpr int kEscapeBudget = 16;
constexpr int kCodebookSize = 15;
constexpr int kEscapeCode = 15;
constexpr uint16_t kNoEscape = 0xFFFF;

// Device status word (bit flags), read back by se12_device_status().
constexpr unsigned kStatusWaitTimeout = 1u;
constexpr unsigned kStatusBadArgument = 2u;

// A wait that has not completed after this many nanoseconds is a logic
// error (a correct wait here completes in microseconds).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// try_wait may suspend the thread up to this long (ns) instead of spinning;
// it returns as soon as the phase completes.
constexpr uint32_t kSuspendHintNs = 1000000u;

// Device status word of the library (one translation unit: se12_lib.cu).
__device__ unsigned int g_status;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void raise_status(unsigned bits) { atomicOr(&g_status, bits); }

// Limit of the waits on other CTAs' and other GPUs' progress (flags,
// counters, epoch-tagged words), in ns: kWaitLimitNs unless the host set
// another (se12_set_wait_limit_ns), e.g. a short one to make a test's wait
// on a peer that never writes run out quickly.
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;

// Such a wait gives up when its limit has passed, or at once when some wait
// already timed out and the host has not cleared the status word: one lost
// peer then ends a kernel after one limit, not one limit per waiting value.
// (Waits for this CTA's own copies, the mbarrier waits, always wait them out.)
__device__ __forceinline__ bool peer_wait_expired(unsigned long long start) {
  if (*reinterpret_cast<volatile unsigned*>(&g_status) & kStatusWaitTimeout) return true;
  return global_ns() - start > *reinterpret_cast<volatile unsigned long long*>(&g_wait_limit_ns);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// Raises the barrier's expected transaction bytes of the current phase
// without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and
// raises kStatusWaitTimeout) if it did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - start > kWaitLimitNs) {
      raise_status(kStatusWaitTimeout);
      return false;
    }
  }
}

// Same, for a warp with nothing else to do: between polls it sleeps with
// exponential backoff (up to ~256 ns) instead of competing for issue slots
// with the warps that share its scheduler.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  unsigned ns = 32;
  while (true) {
    __nanosleep(ns);
    if (mbar_try_wait(bar, parity)) return true;
    if (ns < 256) ns <<= 1;
    if (global_ns() - start > kWaitLimitNs) {
      raise_status(kStatusWaitTimeout);
      return false;
    }
  }
}

// Atomic add on a shared-memory counter with acquire-release semantics at
// CTA scope: orders this thread's earlier shared-memory writes before the
// add, and the later reads after it.
__device__ __forceinline__ int atomic_add_acq_rel_cta(int* counter, int v) {
  int old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(smem_addr(counter)), "r"(v) : "memory");
  return old;
}

// Atomic add on a global counter with acquire-release semantics at GPU
// scope: publishes the calling thread's earlier writes (and, through a
// preceding __syncwarp, its warp's) to whoever acquires a later value, and
// makes writes published by earlier adders visible to the caller.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* counter, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(counter), "r"(v) : "memory");
  return old;
}

// Release store / acquire load of a flag in global memory at GPU scope.
__device__ __forceinline__ void st_release_gpu(int* flag, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* flag) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
  return v;
}

// Waits until *flag is non-zero (acquiring what its writer released).
// Returns false (and raises kStatusWaitTimeout) once peer_wait_expired.
__device__ __forceinline__ bool wait_flag_gpu(const int* flag) {
  if (ld_acquire_gpu(flag)) return true;
  const unsigned long long start = global_ns();
  while (!ld_acquire_gpu(flag)) {
    __nanosleep(64);
    if (peer_wait_expired(start)) {
      raise_status(kStatusWaitTimeout);
      return false;
    }
  }
  return true;
}

// System-scope (all GPUs of the node) release store and acquire load, for
// flags written into another GPU's memory over peer mappings.
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until *flag has reached epoch e (flags only grow; compared modulo
// 2^32). Returns false (and raises kStatusWaitTimeout) once peer_wait_expired.
__device__ __forceinline__ bool wait_epoch_sys(const int* flag, int e) {
  auto reached = [flag, e]() {
    return static_cast<int>(static_cast<unsigned>(ld_acquire_sys(flag)) - static_cast<unsigned>(e)) >= 0;
  };
  if (reached()) return true;
  const unsigned long long start = global_ns();
  while (!reached()) {
    __nanosleep(32);
    if (peer_wait_expired(start)) {
      raise_status(kStatusWaitTimeout);
      return false;
    }
  }
  return true;
}

// 64-bit relaxed stores and loads at system scope: a value and its epoch in
// one naturally aligned word, which a reader sees whole or not at all.
__device__ __forceinline__ void st_word_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_word_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Waits until *p holds epoch e in its high half; returns its low half in
// *value. False (and kStatusWaitTimeout raised) once peer_wait_expired.
__device__ __forceinline__ bool wait_word_sys(const unsigned long long* p, unsigned e, unsigned* value) {
  unsigned long long w = ld_word_sys(p);
  if (static_cast<unsigned>(w >> 32) != e) {
    const unsigned long long start = global_ns();
    do {
      __nanosleep(20);
      if (peer_wait_expired(start)) {
        raise_status(kStatusWaitTimeout);
        return false;
      }
      w = ld_word_sys(p);
    } while (static_cast<unsigned>(w >> 32) != e);
  }
  *value = static_cast<unsigned>(w);
  return true;
}

// ------------------------------------------------------------------ L2 policy

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------------------ TMA

// 2-D tiled tensor load (no multicast) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// 1-D bulk copy global -> shared (no multicast). dst, src 16-byte aligned,
// bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// 3-D tiled tensor load (no multicast).
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Per-thread 16-byte asynchronous copy global -> shared through L2 only.
__device__ __forceinline__ void cp_async_16_cg(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// Same, also caching in L1 (data re-read by this SM).
__device__ __forceinline__ void cp_async_16_ca(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// The mbarrier's pending count is raised by one now and lowered when every
// cp.async this thread issued so far has landed in shared memory.
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Fire-and-forget prefetch of the cache line holding p into L2.
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ------------------------------------------------------------------ PDL

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ named barriers

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------ mma

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------ SE12 decode pieces

// BF16 bits from exponent byte and sign|mantissa byte:
//   bits = ((sm & 0x80) << 8) | (exp << 7) | (sm & 0x7F)
// (the reference's join_bit_pattern, src/lws/domain/weights.py:109-119).
__device__ __forceinline__ uint32_t bf16_bits(uint32_t sm, uint32_t exponent) {
  return ((sm & 0x80u) << 8) | (exponent << 7) | (sm & 0x7Fu);
}

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits) { return __uint_as_float(bits << 16); }

// Pair table entry for one ec byte (two 4-bit codes: even weight in the low
// nibble, odd weight in the high nibble). Entry layout is a BF16x2 word
// holding only the exponent fields (bits 7..14 and 23..30). For the escape
// code the entry instead sets every sign and mantissa bit of that half
// (mask 0x807F); `pair_word` then yields exactly +0.0 for that weight and
// the kernel adds the escaped weight separately.
__device__ __forceinline__ uint32_t pair_entry(const uint8_t* codebook, uint32_t byte) {
  const uint32_t c0 = byte & 0xFu, c1 = byte >> 4;
  const uint32_t h0 = (c0 == kEscapeCode) ? 0x807Fu : (static_cast<uint32_t>(codebook[c0]) << 7);
  const uint32_t h1 = (c1 == kEscapeCode) ? 0x807Fu : (static_cast<uint32_t>(codebook[c1]) << 7);
  return h0 | (h1 << 16);
}

// Combines two sign|mantissa bytes (already placed as [s0,s0,s1,s1]) with a
// pair table entry: keep sign+mantissa bits from `dup` where the entry has
// no kill bits, take the exponent bits from the entry.
//   result = (dup & M & ~entry) | (entry & ~M),  M = 0x807F807F
__device__ __forceinline__ uint32_t pair_word(uint32_t dup, uint32_t entry) {
  uint32_t r;
  // lop3 truth table for f(a=dup, b=entry, c=M) = (a & c & ~b) | (b & ~c) -> 0x2E... computed:
  //   a=0xF0 b=0xCC c=0xAA : (0xF0 & 0xAA & 0x33) | (0xCC & 0x55) = 0x20 | 0x44 = 0x64
  asm("lop3.b32 %0, %1, %2, %3, 0x64;" : "=r"(r) : "r"(dup), "r"(entry), "r"(0x807F807Fu));
  return r;
}

}  // namespace se12
