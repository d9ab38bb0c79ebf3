// Shared device helpers for the MxWave B200 kernels (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mxwave_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "mxwave_b200 kernels target sm_100a only"
#endif

namespace mxw {

constexpr int kBlock = 32;  // MXFP4 block: 32 consecutive input channels share a scale

// ------------------------------------------------------------------ bit utils

__device__ __forceinline__ float bits_f32(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f32_bits(float f) { return __float_as_uint(f); }

// 2^e exactly, for integer e in [-149, 127] (subnormals included).
__device__ __forceinline__ float exp2i(int e) {
  if (e >= -126) return bits_f32(static_cast<uint32_t>(e + 127) << 23);
  return bits_f32(1u << (e + 149));
}

// floor() and ceil() of torch.log2 on an fp32 value q > 0 (normal).
// torch's fp32 log2 equals the double log2 rounded to fp32; that rounding can
// only move the result onto an integer when q's significand is within 256 ulps
// of 2 (floor) or of 1 (ceil), so only those cases evaluate the double log2.
__device__ __forceinline__ int floor_log2_f32(float q) {
  uint32_t b = f32_bits(q);
  int e = static_cast<int>((b >> 23) & 0xff) - 127;
  uint32_t man = b & 0x7fffffu;
  if (man >= 0x7fff00u) return static_cast<int>(floorf(__double2float_rn(log2(static_cast<double>(q)))));
  return e;
}

__device__ __forceinline__ int ceil_log2_f32(float q) {
  uint32_t b = f32_bits(q);
  int e = static_cast<int>((b >> 23) & 0xff) - 127;
  uint32_t man = b & 0x7fffffu;
  if (man == 0) return e;
  if (man < 0x100u) return static_cast<int>(ceilf(__double2float_rn(log2(static_cast<double>(q)))));
  return e + 1;
}

// ------------------------------------------------------------ packed f32x2 ops
// sm_100 executes these as single FMUL2/FFMA2/FADD2 instructions; each lane is
// an ordinary IEEE fp32 operation with round-to-nearest-even (no contraction).

struct f2 {
  float x, y;
};

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  return (static_cast<unsigned long long>(f32_bits(hi)) << 32) | f32_bits(lo);
}
__device__ __forceinline__ f2 unpack2(unsigned long long v) {
  return f2{bits_f32(static_cast<uint32_t>(v)), bits_f32(static_cast<uint32_t>(v >> 32))};
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b,
                                                   unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Correctly rounded packed product for a result that feeds an addition.
// ptxas contracts "mul.rn.f32x2 -> add.rn.f32x2" into a single fma even with
// the explicit rounding modifier (measured on sm_100a), which would skip the
// product's rounding.  An fma with a -0 addend rounds exactly like the
// multiply (a*b + -0 == a*b, signed zeros included) and leaves nothing to
// contract.  `nz2` must be -0.0 in both halves and come from a runtime value
// (a kernel argument), so the compiler cannot rewrite the fma as a multiply.
__device__ __forceinline__ unsigned long long mul2_rounded(unsigned long long a, unsigned long long b,
                                                           unsigned long long nz2) {
  return fma2(a, b, nz2);
}

// ----------------------------------------------------------------- E2M1 codes

// Two fp32 values -> one byte of E2M1 codes, `lo` in bits 0-3 and `hi` in bits
// 4-7, rounded to nearest with ties to even and saturated to +-6 (the
// reference's clamp(-6, 6) followed by its tie-to-even bucket rule).
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

// Two non-negative E2M1 codes (0..7, one per nibble of `byte`) -> their
// magnitudes as an fp32 pair, through two byte permutes: the f16 encodings of
// {0, 0.5, 1, 1.5, 2, 3, 4, 6} differ only in their high byte, so a byte
// table lookup yields an exact f16x2 that converts to fp32 exactly.
__device__ __forceinline__ unsigned long long e2m1_mag_to_f32x2(uint32_t byte) {
  const uint32_t u = __byte_perm(0x3E3C3800u, 0x46444240u, byte);  // [HB[c0], HB[c1], 0, 0]
  uint32_t h = __byte_perm(u, 0u, 0x1404u);                         // [0, HB[c0], 0, HB[c1]]
  const __half2 hh = *reinterpret_cast<__half2*>(&h);
  return pack2(__low2float(hh), __high2float(hh));
}

// Signed E2M1 codes (one per nibble) -> signed fp32 magnitudes (dequantisation).
__device__ __forceinline__ unsigned long long e2m1x2_to_f32x2(uint32_t byte) {
  const unsigned long long m = e2m1_mag_to_f32x2(byte & 0x77u);
  const uint32_t s0 = (byte & 0x08u) << 28, s1 = (byte & 0x80u) << 24;
  return m ^ ((static_cast<unsigned long long>(s1) << 32) | s0);
}

}  // namespace mxw
