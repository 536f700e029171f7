// Shared device helpers: mbarriers, bulk async copies, byte extraction.  The
// kernels bound every wait by wall-clock time (%globaltimer, gemv.cuh
// wait_phase), not by a poll count.  Everything here targets sm_100a only.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#ifndef FRC_DEVICE_INLINE
#define FRC_DEVICE_INLINE __device__ __forceinline__
#endif

namespace frc {

// Bits of the per-device status word (frc_device_status).
enum : uint32_t {
  kStatusFullWaitTimeout  = 1u << 0,  // a consumer gave up waiting for a tile
  kStatusEmptyWaitTimeout = 1u << 1,  // the producer gave up waiting for a free stage
  kStatusDrainTimeout     = 1u << 2,  // the producer gave up draining its copies
  kStatusSmemMisaligned   = 1u << 3,  // dynamic shared memory not 128-byte aligned (kernel skipped)
  kStatusGatherTimeout    = 1u << 4,  // a fused all-gather wait gave up on a rank's flag
};

FRC_DEVICE_INLINE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

FRC_DEVICE_INLINE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

FRC_DEVICE_INLINE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

FRC_DEVICE_INLINE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

FRC_DEVICE_INLINE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

FRC_DEVICE_INLINE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// 1-D bulk copy global -> shared, completion signalled on `bar` as tx bytes.
// dst, src 16-byte aligned; bytes a nonzero multiple of 16.
FRC_DEVICE_INLINE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

FRC_DEVICE_INLINE void named_barrier_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

FRC_DEVICE_INLINE float half_bits_to_float(uint32_t h16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xFFFFu)));
}

// Little-endian 16-bit value at a 2-byte aligned address.
FRC_DEVICE_INLINE uint32_t ld_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

// Four bytes starting at a 2-byte aligned address p, as one little-endian
// word; reads only the aligned words overlapping [p, p+4).
FRC_DEVICE_INLINE uint32_t ld_u32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if ((a & 3u) == 0) return *reinterpret_cast<const uint32_t*>(p);
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return static_cast<uint32_t>(q[0]) | (static_cast<uint32_t>(q[1]) << 16);
}

// N little-endian words starting at a 2-byte aligned shared-memory address,
// via N+1 aligned 32-bit loads and funnel shifts (no divergence on the
// alignment).  The bytes [p - 2, p + 4N + 2) must lie inside the buffer.
template <int N>
FRC_DEVICE_INLINE void lds_words_a2(const uint8_t* p, uint32_t (&out)[N]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
  uint32_t w[N + 1];
#pragma unroll
  for (int i = 0; i <= N; ++i) w[i] = base[i];
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// Shared-memory loads at a 32-bit shared address plus an immediate byte
// offset (one LDS each, no generic-address arithmetic).  Volatile keeps them
// after the mbarrier waits that publish the stage they read.
template <int OFF>
FRC_DEVICE_INLINE uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+%5];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a), "n"(OFF));
  return v;
}
template <int OFF>
FRC_DEVICE_INLINE uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
  return v;
}
template <int OFF>
FRC_DEVICE_INLINE uint32_t lds16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1+%2];" : "=h"(v) : "r"(a), "n"(OFF));
  return v;
}

// N little-endian words starting OFF bytes past the 4-byte aligned shared
// address a, shifted right by sh bits (0 or 16) across word boundaries: the N
// words at byte a + OFF + sh / 8.  Reads the words [a + OFF, a + OFF + 4N + 4).
template <int N, int OFF>
FRC_DEVICE_INLINE void lds_words_sh(uint32_t a, uint32_t sh, uint32_t (&out)[N]) {
  uint32_t w[N + 1];
  if constexpr (N >= 1) w[0] = lds32<OFF>(a);
  if constexpr (N >= 1) w[1] = lds32<OFF + 4>(a);
  if constexpr (N >= 2) w[2] = lds32<OFF + 8>(a);
  if constexpr (N >= 3) w[3] = lds32<OFF + 12>(a);
  if constexpr (N >= 4) w[4] = lds32<OFF + 16>(a);
  if constexpr (N >= 5) w[5] = lds32<OFF + 20>(a);
  if constexpr (N >= 6) w[6] = lds32<OFF + 24>(a);
  if constexpr (N >= 7) w[7] = lds32<OFF + 28>(a);
  if constexpr (N >= 8) w[8] = lds32<OFF + 32>(a);
  static_assert(N <= 8, "at most 8 words");
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// Byte b (0..3) of word w placed as the mantissa byte of 1.0f:
// returns 1 + ((w >> 8b) & 0xFF) / 128 for bytes already ORed with 0x80,
// i.e. the float 0x3F80_0000 | (low 7 bits << 16).
template <int B>
FRC_DEVICE_INLINE float byte_as_unit_float(uint32_t w) {
  // selector: out byte3 = 0x3F (b.byte3), byte2 = w.byteB, bytes1,0 = 0.
  constexpr uint32_t sel = 0x7000u | (static_cast<uint32_t>(B) << 8) | 0x44u;
  return __uint_as_float(__byte_perm(w, 0x3F000000u, sel));
}

// Byte b of w as the low mantissa byte of 2^23: returns 2^23 + byte.
template <int B>
FRC_DEVICE_INLINE float byte_as_magic_float(uint32_t w) {
  constexpr uint32_t sel = 0x7650u | static_cast<uint32_t>(B);
  return __uint_as_float(__byte_perm(w, 0x4B000000u, sel));
}

FRC_DEVICE_INLINE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace frc
