// Kernels and launchers of K1, the MXFP4 quantizer (see quantize.cu for the
// algorithm).  Included by one translation unit per input type
// (quantize_bf16.cu, quantize_f16.cu, quantize_f32.cu), which instantiate the
// launchers for that type in parallel builds.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "runtime.h"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace mxw {

constexpr int kTileRows = 32;
constexpr int kTileBlocks = 8;
constexpr int kConsumerWarps = kTileBlocks;
constexpr int kProducerWarp = kConsumerWarps;      // TMA loads
constexpr int kStoreWarp = kConsumerWarps + 1;     // TMA stores of packed bytes + scale rows
constexpr int kQuantThreads = (kConsumerWarps + 2) * 32;
constexpr int kStages = 4;
constexpr int kBoxBytes = kTileRows * 128;  // one TMA box: 32 rows x 128 bytes
constexpr int kOutTileBytes = kTileRows * kTileBlocks * 16;  // packed bytes of one tile (32 x 128)
constexpr int kScaleTileBytes = kTileRows * kTileBlocks;      // scale bytes of one tile (32 x 8)
// Output staging ring: consumers fill a buffer and arrive on out_full; the store
// warp writes it out and, once the TMA store no longer reads it, arrives on
// out_empty.  No barrier couples the consumer warps to each other.
constexpr int kOutBuffers = 4;

enum Obj { kObjNone = 0, kObjGamma = 1, kObjHess = 2, kObjRtn = 3 };
enum QMode { kQAmax = 0, kQTop2 = 1, kQGeneral = 2 };

struct QuantParams {
  int64_t rows, cols, nb, n_row_tiles, n_tiles;
  const void* weight;  // the input again, for the rare blocks re-read from global memory
  int64_t ld;
  const float* gamma;
  const float* hessian;
  uint8_t* packed;
  uint8_t* scales;
  uint32_t* flags;
  int depth;
  int q_below, q_above, q_small;
  float q_w;
  // Always 0.0f.  Added to the scaled values before encoding so that -0
  // becomes +0 (code 0, as the reference's "scaled < 0" sign rule gives); a
  // runtime operand keeps the compiler from folding "x + 0" into "x".
  float zero;
  // Always -0.0f: the addend of mul2_rounded (see common.cuh).
  float negzero;
};

template <int DT>
struct Elem {
  static constexpr int kBytes = DT == MXW_F32 ? 4 : 2;
  static constexpr int kBoxCols = 128 / kBytes;
  static constexpr int kBoxesPerStage = kTileBlocks * kBlock * kBytes / 128;
  static constexpr int kStageBytes = kBoxesPerStage * kBoxBytes;
};

// Everything a thread knows about its block after loading it.  2-byte inputs
// keep their raw words (16 registers); fp32 inputs keep the signed pairs.
// Both keep nt2 = -|t| as fp32 pairs (elements 2j, 2j+1), the input of the
// error evaluation.
template <int DT>
struct BlockData {
  static constexpr bool kWords = DT != MXW_F32;
  uint32_t words[kWords ? 16 : 1];
  unsigned long long t2[kWords ? 1 : 16];
  unsigned long long nt2[16];
  float amax, second;  // largest / second-largest magnitude
  bool nonfinite;

  // Signed element pair j as fp32.
  __device__ __forceinline__ unsigned long long signed_pair(int j) const {
    if constexpr (DT == MXW_BF16) {
      return pack2(bits_f32(words[j] << 16), bits_f32(words[j] & 0xffff0000u));
    } else if constexpr (DT == MXW_F16) {
      const __half2 h = *reinterpret_cast<const __half2*>(&words[j]);
      return pack2(__low2float(h), __high2float(h));
    } else {
      return t2[j];
    }
  }
  // Sign bits of element pair j, positioned as fp32 sign bits of a pair.
  __device__ __forceinline__ unsigned long long sign_pair(int j) const {
    if constexpr (kWords) {
      return (static_cast<unsigned long long>(words[j] & 0x80000000u) << 32) |
             static_cast<unsigned long long>((words[j] & 0x8000u) << 16);
    } else {
      return t2[j] & 0x8000000080000000ull;
    }
  }
};

__device__ __forceinline__ unsigned long long neg_abs2(unsigned long long v) {
  return v | 0x8000000080000000ull;
}

// ------------------------------------------------------------ block loading

template <int DT, int QM>
__device__ __forceinline__ void finish_stats_16bit(BlockData<DT>& B) {
  // Magnitude order statistics on the raw 16-bit patterns (sign-magnitude:
  // the integer order of |bits| is the order of |value|; NaN/inf on top).
  uint32_t m1 = 0, m2 = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const uint32_t a = B.words[k] & 0x7fff7fffu;
    if constexpr (QM == kQTop2) m2 = __vmaxu2(m2, __vminu2(m1, a));
    m1 = __vmaxu2(m1, a);
  }
  const uint32_t lo1 = m1 & 0xffffu, hi1 = m1 >> 16;
  const uint32_t top1 = max(lo1, hi1);
  uint32_t top2 = 0;
  if constexpr (QM == kQTop2) top2 = max(min(lo1, hi1), max(m2 & 0xffffu, m2 >> 16));
  if constexpr (DT == MXW_BF16) {
    B.nonfinite = top1 >= 0x7f80u;
    B.amax = bits_f32(top1 << 16);
    B.second = bits_f32(top2 << 16);
  } else {
    B.nonfinite = top1 >= 0x7c00u;
    B.amax = __half2float(__ushort_as_half(static_cast<unsigned short>(top1)));
    B.second = __half2float(__ushort_as_half(static_cast<unsigned short>(top2)));
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) B.nt2[k] = neg_abs2(B.signed_pair(k));
}

template <int DT, int QM>
__device__ __forceinline__ void finish_stats_f32(BlockData<DT>& B, const unsigned long long (&t2)[16]) {
  uint32_t m1 = 0, m2 = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const f2 v = unpack2(t2[j]);
    const uint32_t a0 = f32_bits(v.x) & 0x7fffffffu, a1 = f32_bits(v.y) & 0x7fffffffu;
    if constexpr (QM == kQTop2) m2 = max(m2, min(m1, a0));
    m1 = max(m1, a0);
    if constexpr (QM == kQTop2) m2 = max(m2, min(m1, a1));
    m1 = max(m1, a1);
    B.nt2[j] = neg_abs2(t2[j]);
  }
  B.nonfinite = m1 >= 0x7f800000u;
  B.amax = bits_f32(m1);
  B.second = bits_f32(m2);
}

// The 16 words (32 two-byte elements) of the block in tile row `lane`, block
// column `w`, from a 128B-swizzled stage.
__device__ __forceinline__ void stage_words(const uint8_t* stage, int w, int lane, uint32_t (&words)[16]) {
  const uint8_t* box = stage + (w >> 1) * kBoxBytes + lane * 128;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = (4 * (w & 1) + j) ^ (lane & 7);
    const uint4 v = *reinterpret_cast<const uint4*>(box + (c << 4));
    words[4 * j + 0] = v.x;
    words[4 * j + 1] = v.y;
    words[4 * j + 2] = v.z;
    words[4 * j + 3] = v.w;
  }
}

// Signed element pair of a word of two 2-byte elements, as fp32.
template <int DT>
__device__ __forceinline__ unsigned long long word_pair(uint32_t w) {
  if constexpr (DT == MXW_BF16) {
    return pack2(bits_f32(w << 16), bits_f32(w & 0xffff0000u));
  } else {
    const __half2 h = *reinterpret_cast<const __half2*>(&w);
    return pack2(__low2float(h), __high2float(h));
  }
}

// Read this thread's block (row `lane` of the tile, block column `w`) from a
// swizzled stage.
template <int DT, int QM>
__device__ __forceinline__ void read_block_smem(const uint8_t* stage, int w, int lane, BlockData<DT>& B) {
  if constexpr (Elem<DT>::kBytes == 2) {
    stage_words(stage, w, lane, B.words);
    finish_stats_16bit<DT, QM>(B);
  } else {
    const uint8_t* box = stage + w * kBoxBytes + lane * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 v = *reinterpret_cast<const float4*>(box + ((c ^ (lane & 7)) << 4));
      B.t2[2 * c] = pack2(v.x, v.y);
      B.t2[2 * c + 1] = pack2(v.z, v.w);
    }
    finish_stats_f32<DT, QM>(B, B.t2);
  }
}

// k-th smallest magnitude (0-based) of the block, by rank counting.
__device__ __forceinline__ float kth_magnitude(const unsigned long long (&nt2)[16], int k) {
  float a[32];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const f2 v = unpack2(nt2[j]);
    a[2 * j] = -v.x;
    a[2 * j + 1] = -v.y;
  }
  float result = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    int lt = 0, le = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      lt += a[j] < a[i];
      le += a[j] <= a[i];
    }
    if (lt <= k && k < le) result = a[i];
  }
  return result;
}

// ------------------------------------------------------------- error kernels

// |dW| for one element pair: q(|t| / 2^e) * 2^e - |t|, with nt = -|t|.  The
// product q*2^e is exact, so the fused form rounds like the reference's
// separate multiply and subtract, except when q*2^e overflows (e >= 126),
// which takes the unfused path.
template <bool UNFUSED>
__device__ __forceinline__ unsigned long long abs_dw2(unsigned long long nt, unsigned long long NI2,
                                                      unsigned long long S2, unsigned long long NZ2) {
  const f2 x = unpack2(mul2(nt, NI2));  // |t| / 2^e exactly (NI2 = -2^-e)
  uint32_t h2;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
      : "=r"(h2) : "f"(x.y), "f"(x.x));
  const __half2 hh = *reinterpret_cast<const __half2*>(&h2);
  const unsigned long long q = pack2(__low2float(hh), __high2float(hh));
  if constexpr (UNFUSED) return add2(mul2_rounded(q, S2, NZ2), nt);
  return fma2(q, S2, nt);
}

// Unweighted / gamma error of one candidate exponent e: mean over the block of
// dW^2 (times gamma^2), core.py:224-234.
// gamma^2 pair j of the warp's block column from shared memory (every lane
// reads the same address: a broadcast).  Volatile, so the loads stay inside
// the candidate loop instead of being hoisted into 32 registers.
__device__ __forceinline__ unsigned long long load_g2(const float* Gw, int j) {
  unsigned long long v;
  asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v) : "r"(smem_u32(Gw + 2 * j)));
  return v;
}

// GS: gamma^2 pairs from shared memory (Gw) instead of registers (g2).
template <bool GAMMA, bool UNFUSED, bool GS = false>
__device__ __forceinline__ float candidate_error(const unsigned long long (&nt2)[16], int e,
                                                 const unsigned long long (&g2)[16], unsigned long long NZ2,
                                                 const float* Gw = nullptr) {
  const float s = exp2i(e);
  const float ninv = -exp2i(-e);
  const unsigned long long S2 = pack2(s, s), NI2 = pack2(ninv, ninv);
  unsigned long long p[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int lp = 0; lp < 4; ++lp) {
      const int j = q * 4 + lp;
      const unsigned long long d = abs_dw2<UNFUSED>(nt2[j], NI2, S2, NZ2);
      // fl(dW^2), then fl(fl(dW^2) * gamma^2): each product rounded before the add.
      unsigned long long sq = mul2_rounded(d, d, NZ2);
      if constexpr (GAMMA) sq = mul2_rounded(sq, GS ? load_g2(Gw, j) : g2[j], NZ2);
      p[lp] = (q == 0) ? sq : add2(p[lp], sq);
    }
  }
  float acc = unpack2(p[0]).x;
  acc = __fadd_rn(acc, unpack2(p[0]).y);
#pragma unroll
  for (int lp = 1; lp < 4; ++lp) {
    const f2 v = unpack2(p[lp]);
    acc = __fadd_rn(acc, v.x);
    acc = __fadd_rn(acc, v.y);
  }
  return __fmul_rn(acc, 0.03125f);
}

// Block-Hessian error of one candidate: sum_d (sum_s dW_s H[s,d]) dW_d with
// the inner sum as a sequential fp32 FMA chain over s (core.py:228-229).
// dW = sign(t) * |dW| (sign bit transferred exactly); dW pairs are rebuilt on
// the fly instead of being held in 32 registers.
// One 16-byte row fragment of the block Hessian.  Volatile loads: H is the
// same for every candidate, and letting the compiler hoist all 256 fragments
// out of the candidate loop would spill them to local memory.
template <bool SHARED>
__device__ __forceinline__ ulonglong2 load_h16(const float* p) {
  ulonglong2 v;
  if constexpr (SHARED) {
    asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "r"(smem_u32(p)));
  } else {
    asm volatile("ld.global.nc.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p));
  }
  return v;
}

template <int DT, bool HS_SHARED, bool UNFUSED>
__device__ __forceinline__ float candidate_error_hessian(const BlockData<DT>& B, int e, const float* Hs,
                                                         unsigned long long NZ2) {
  const float s = exp2i(e);
  const float ninv = -exp2i(-e);
  const unsigned long long S2 = pack2(s, s), NI2 = pack2(ninv, ninv);
  unsigned long long w[16];
#pragma unroll
  for (int sp = 0; sp < 16; ++sp) {
    const f2 d = unpack2(abs_dw2<UNFUSED>(B.nt2[sp], NI2, S2, NZ2) ^ B.sign_pair(sp));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int si = 2 * sp + h;
      const float dv = h ? d.y : d.x;
      const unsigned long long ds = pack2(dv, dv);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const ulonglong2 hv = load_h16<HS_SHARED>(Hs + si * 32 + 4 * k);
        if (si == 0) {
          w[2 * k] = mul2(ds, hv.x);
          w[2 * k + 1] = mul2(ds, hv.y);
        } else {
          w[2 * k] = fma2(ds, hv.x, w[2 * k]);
          w[2 * k + 1] = fma2(ds, hv.y, w[2 * k + 1]);
        }
      }
    }
  }
  unsigned long long p[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int lp = 0; lp < 4; ++lp) {
      const int j = q * 4 + lp;
      const unsigned long long d = abs_dw2<UNFUSED>(B.nt2[j], NI2, S2, NZ2) ^ B.sign_pair(j);
      const unsigned long long prod = mul2_rounded(w[j], d, NZ2);
      p[lp] = (q == 0) ? prod : add2(p[lp], prod);
    }
  }
  float acc = unpack2(p[0]).x;
  acc = __fadd_rn(acc, unpack2(p[0]).y);
#pragma unroll
  for (int lp = 1; lp < 4; ++lp) {
    const f2 v = unpack2(p[lp]);
    acc = __fadd_rn(acc, v.x);
    acc = __fadd_rn(acc, v.y);
  }
  return acc;
}

// _rtn_scale_exponent (core.py:91-104).
__device__ __forceinline__ int rtn_exponent(float block_max) {
  if (!(block_max > 0.0f)) return -127;
  const float safe = fmaxf(block_max, 1.17549435e-38f);
  const int base = floor_log2_f32(safe);
  const float sig = __fdiv_rn(safe, exp2i(base));
  return base + (sig >= 1.75f ? 1 : 0) - 2;
}

// ------------------------------------------------------------- block driver

// Chooses the exponent and encodes one block into 16 packed bytes; returns the
// E8M0 byte.  `Hs`: the block's Hessian (shared or global memory) or unused.
// FAST (unweighted / gamma objectives of the TMA kernel): the candidate loop
// carries only the fused error form.  A block with a candidate e >= 126,
// where q * 2^e can overflow (largest magnitude near FLT_MAX), is left for
// quantize_fixup_kernel: it gets the marker scale byte kRareBlock, which no
// quantized block can have (scale bytes are 0..254).  Keeping the rare form
// out of the hot loop saves registers and instructions there (5-7 % of
// kernel time on B200).
constexpr uint32_t kRareBlock = 255;

// Final encode (core.py:242-249): x = clamp(t / 2^raw) -> nibble, -0 -> code 0.
// `pair(j)` yields the signed element pair j as fp32.
template <typename PairFn>
__device__ __forceinline__ void encode_pairs(PairFn pair, const QuantParams& P, int raw, uint4& packed) {
  const float inv = exp2i(-raw);
  const unsigned long long I2 = pack2(inv, inv);
  const unsigned long long Z2 = pack2(P.zero, P.zero);
  const unsigned long long NZ2e = pack2(P.negzero, P.negzero);
  uint32_t bytes[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const f2 x = unpack2(add2(mul2_rounded(pair(j), I2, NZ2e), Z2));
    bytes[j] = e2m1x2(x.x, x.y);
  }
  packed.x = __byte_perm(__byte_perm(bytes[0], bytes[1], 0x0040), __byte_perm(bytes[2], bytes[3], 0x0040), 0x5410);
  packed.y = __byte_perm(__byte_perm(bytes[4], bytes[5], 0x0040), __byte_perm(bytes[6], bytes[7], 0x0040), 0x5410);
  packed.z = __byte_perm(__byte_perm(bytes[8], bytes[9], 0x0040), __byte_perm(bytes[10], bytes[11], 0x0040), 0x5410);
  packed.w =
      __byte_perm(__byte_perm(bytes[12], bytes[13], 0x0040), __byte_perm(bytes[14], bytes[15], 0x0040), 0x5410);
}

template <int DT>
__device__ __forceinline__ void encode_block(const BlockData<DT>& B, const QuantParams& P, int raw, uint4& packed) {
  encode_pairs([&](int j) { return B.signed_pair(j); }, P, raw, packed);
}

// The percentile anchor of a block (core.py:183-189): amax, or torch.quantile
// by linear interpolation between two order statistics.
template <int QM>
__device__ __forceinline__ float block_anchor(float amax, float second, const unsigned long long (&nt2)[16],
                                              const QuantParams& P) {
  if constexpr (QM == kQAmax) {
    return amax;
  } else {
    float lo, hi;
    if constexpr (QM == kQTop2) {
      lo = P.q_below == 31 ? amax : second;
      hi = P.q_above == 31 ? amax : second;
    } else {
      lo = kth_magnitude(nt2, P.q_below);
      hi = (P.q_above == P.q_below) ? lo : kth_magnitude(nt2, P.q_above);
    }
    const float d = __fsub_rn(hi, lo);
    return P.q_small ? __fmaf_rn(P.q_w, d, lo) : __fmaf_rn(__fsub_rn(P.q_w, 1.0f), d, hi);
  }
}

// floor(torch.log2(x / 6)) and ceil(torch.log2(y / 6)) in fp32 for finite
// x >= 1e-6 and y >= 1e-12, without the division.  With x = m * 2^E, fl(x/6)
// lies in [2^(E-2), 2^(E-1)) for m >= 1.5 and in (2^(E-3), 2^(E-2)) below
// (the rounded quotient never reaches the power of two).  torch's fp32 log2
// can round to an integer only when the quotient is within 256 ulps of a
// power of two: for floor that is m within 256 ulps under 1.5, for ceil m
// within 512 ulps over 1.5; those take the division and the exact test.
// Agreement with the division-based definition outside the bands was checked
// on the CPU for every fp32 value in range (oracle/check_exponents.c).
__device__ __forceinline__ int floor_log2_div6(float x) {
  const uint32_t b = f32_bits(x);
  const uint32_t man = b & 0x7fffffu;
  if (man - (0x400000u - 256u) < 256u || b >= 0x7f800000u) return floor_log2_f32(__fdiv_rn(x, 6.0f));
  return static_cast<int>(b >> 23) - 127 - (man >= 0x400000u ? 2 : 3);
}

__device__ __forceinline__ int ceil_log2_div6(float y) {
  const uint32_t b = f32_bits(y);
  const uint32_t man = b & 0x7fffffu;
  if (man - 0x400001u < 512u || b >= 0x7f800000u) return ceil_log2_f32(__fdiv_rn(y, 6.0f));
  return static_cast<int>(b >> 23) - 127 - (man > 0x400000u ? 1 : 2);
}

template <int DT, int OBJ, int QM, bool HS_SHARED, bool GS = false, bool FAST = false>
__device__ __forceinline__ uint32_t quantize_one_block(const BlockData<DT>& B, const QuantParams& P,
                                                       const unsigned long long (&g2)[16], const float* Hs,
                                                       uint4& packed, const float* Gw = nullptr) {
  int raw;
  bool rare = false;  // FAST only: a candidate e >= 126 -> left for quantize_fixup_kernel
  if constexpr (OBJ == kObjRtn) {
    // core.py:240-243: the exponent is clamped to [-127, 127] before storage.
    // An infinite maximum gives log2 = inf there, clamped to 127; a NaN
    // maximum fails the `> 0` test and gives -127 (rtn_exponent).
    raw = isinf(B.amax) ? 127 : max(-127, min(127, rtn_exponent(B.amax)));
  } else {
    float anchor = block_anchor<QM>(B.amax, B.second, B.nt2, P);
    // Non-finite blocks, as the reference's float arithmetic takes them
    // (core.py:183-249): torch.quantile is NaN when the block holds a NaN, and
    // its lerp turns an infinity into NaN for w >= 0.5.  A NaN anchor makes
    // every candidate NaN, so the exponent stays NaN: its E8M0 byte is the
    // x86 float->uint8 conversion of NaN (0) and every scaled value is NaN,
    // which the bucket search maps to code 7 with no sign.  An infinite anchor
    // makes every candidate +inf, clamped to 127.
    if (isnan(B.amax) || isnan(anchor)) {
      packed = make_uint4(0x77777777u, 0x77777777u, 0x77777777u, 0x77777777u);
      return 0u;
    }
    if (isinf(anchor)) {
      encode_block(B, P, 127, packed);
      return 254u;
    }
    const bool near_zero = B.amax < 1e-6f;
    anchor = fmaxf(anchor, 1e-6f);
    const int floor_e = floor_log2_div6(anchor);
    const int lo_e = max(-127, min(127, floor_e - P.depth));
    if (near_zero) {
      // t is replaced by zeros (core.py:194-195): every candidate has error 0,
      // the first candidate wins the strict-< argmin and every code is 0.
      packed = make_uint4(0u, 0u, 0u, 0u);
      return static_cast<uint32_t>(lo_e + 127);
    }
    const int hi_e = max(-127, min(127, floor_e + 1));
    const int safe_e = max(-127, min(127, ceil_log2_div6(fmaxf(B.amax, 1e-12f))));
    const unsigned long long NZ2 = pack2(P.negzero, P.negzero);
    float best = __int_as_float(0x7f800000);
    raw = lo_e;
    // Candidates floor-depth .. floor+1 (clamped: equal neighbours are skipped,
    // their error would be identical and never strictly smaller), then the
    // no-clipping exponent unless it repeats one of them.
    const int n_seq = hi_e - lo_e + 1;
    const bool safe_new = safe_e < lo_e || safe_e > hi_e;
    if constexpr (FAST) {
      // No early exit (it would split the hot path): the block runs on with
      // the fused form and only its scale byte becomes the marker.
      rare = (safe_new ? max(hi_e, safe_e) : hi_e) >= 126;
    }
    for (int k = 0; k < n_seq + (safe_new ? 1 : 0); ++k) {
      const int e = k < n_seq ? lo_e + k : safe_e;
      // q * 2^e can overflow only for e >= 126: that rare case takes the
      // unfused multiply-then-subtract form (a block-uniform branch).
      float err;
      if constexpr (OBJ == kObjHess) {
        err = e < 126 ? candidate_error_hessian<DT, HS_SHARED, false>(B, e, Hs, NZ2)
                      : candidate_error_hessian<DT, HS_SHARED, true>(B, e, Hs, NZ2);
      } else {
        if constexpr (FAST) {
          err = candidate_error<OBJ == kObjGamma, false, GS>(B.nt2, e, g2, NZ2, Gw);
        } else {
          err = e < 126 ? candidate_error<OBJ == kObjGamma, false, GS>(B.nt2, e, g2, NZ2, Gw)
                        : candidate_error<OBJ == kObjGamma, true, GS>(B.nt2, e, g2, NZ2, Gw);
        }
      }
      if (err < best) raw = e;
      best = (isnan(err) || isnan(best)) ? __int_as_float(0x7fffffff) : fminf(best, err);
    }
  }
  encode_block(B, P, raw, packed);
  if constexpr (OBJ == kObjRtn) {
    if (isnan(B.amax)) {
      // NaN elements of an rtn block: the reference's bucket search puts a NaN
      // in bucket 7 and its sign test (x < 0) is false, so the code is 7
      // whatever the hardware conversion does with a NaN.
      uint32_t w[4] = {packed.x, packed.y, packed.z, packed.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const f2 v = unpack2(B.signed_pair(j));
        uint32_t& word = w[j >> 2];
        const int sh = 8 * (j & 3);
        if (isnan(v.x)) word = (word & ~(0xfu << sh)) | (0x7u << sh);
        if (isnan(v.y)) word = (word & ~(0xf0u << sh)) | (0x70u << sh);
      }
      packed = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  return rare ? kRareBlock : static_cast<uint32_t>(raw + 127);
}

// Per-warp block-column state in shared memory: gamma^2 (fp32, then the same
// values as bf16x2 pairs for the clipping bound) or the block Hessian.
constexpr int kGammaWords = kBlock + kBlock / 2;

template <int OBJ>
__device__ __forceinline__ void load_column_state(const QuantParams& P, int64_t b, int lane, float* Hw, float* Gw) {
  if constexpr (OBJ == kObjGamma) {
    __syncwarp();
    const float g = __ldg(P.gamma + b * kBlock + lane);
    const float g2 = __fmul_rn(g, g);
    Gw[lane] = g2;
    const float g2n = __shfl_down_sync(0xffffffffu, g2, 1);
    if ((lane & 1) == 0) {
      uint32_t pr;
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pr) : "f"(g2n), "f"(g2));
      reinterpret_cast<uint32_t*>(Gw + kBlock)[lane >> 1] = pr;
    }
    __syncwarp();
  }
  if constexpr (OBJ == kObjHess) {
    __syncwarp();
    const float4* src = reinterpret_cast<const float4*>(P.hessian + b * 1024);
#pragma unroll
    for (int j = 0; j < 8; ++j) reinterpret_cast<float4*>(Hw)[lane + 32 * j] = __ldg(src + lane + 32 * j);
    __syncwarp();
  }
}

// ------------------------------------------------ two-candidate fast path
//
// 2-byte inputs, top-2 or amax anchor.  The reference's candidate order is
// f-depth, ..., f-1, f, f+1 and then the no-clipping exponent `safe` when it
// is new (core.py:201-209).  With an anchor at or below the block maximum,
// safe >= f, so it is new only as f+2 or higher.  Each thread evaluates its
// own block's f and f+1 errors exactly, in one pass that also yields each
// candidate's codes.  The clipping candidates below f are dropped when a lower
// bound on the error of f-1 certifiably exceeds min(E_f, E_f+1): the bound
// grows as the clip threshold falls, so it covers every deeper candidate too,
// and a strictly larger error never wins the strict-< argmin.  Only warps with
// a block the bound does not decide (none unweighted on normal weights, about
// a quarter with gamma weights), or with a block whose safe exponent is f+2,
// evaluate those extra candidates, each thread for its own block.  Blocks
// outside the path's
// preconditions (non-finite values, block scales of 2^15 and above,
// safe >= f+3, NaN errors) take the rare marker and are finished by
// quantize_fixup_kernel.

template <int DT, int OBJ, int QM>
struct FastPath {
  static constexpr bool value =
      Elem<DT>::kBytes == 2 && (OBJ == kObjNone || OBJ == kObjGamma) && (QM == kQTop2 || QM == kQAmax);
};

__device__ __forceinline__ float nan_min(float best, float err) {
  return (isnan(err) || isnan(best)) ? __int_as_float(0x7fffffff) : fminf(best, err);
}

// Certified "E_{f-1} > E_hi" from a computed lower bound `lb` of E_{f-1}.
// lb is at most 1.09x the exact sum it bounds (at most 21 roundings of 2^-8
// each in bf16 arithmetic; fp32 is tighter) and the reference's fp32 error is
// at least (1 - 2^-20)x the exact sum once it is far above the subnormal
// range, so 7/8 of lb is a strict lower bound there.
__device__ __forceinline__ bool lb_prunes(float lb, float e_hi) {
  const float l = __fmul_rn(lb, 0.875f);
  return l > e_hi && l >= 0x1p-100f && lb < __int_as_float(0x7f800000);
}

// sum over the block of g2_i * max(|t_i| - c, 0)^2, in bf16x2 arithmetic
// (bf16 inputs).  c = 3 * 2^f has two significant bits, so -c is exact in bf16.
template <bool GAMMA>
__device__ __forceinline__ float clip_excess_bf16(const uint32_t (&words)[16], float c, const uint32_t* G2b) {
  const uint32_t nc = (f32_bits(-c) >> 16) * 0x00010001u;
  const uint32_t one = 0x3f803f80u;
  uint32_t acc = 0u;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t a = words[j] & 0x7fff7fffu;
    uint32_t v;
    asm("fma.rn.relu.bf16x2 %0, %1, %2, %3;" : "=r"(v) : "r"(a), "r"(one), "r"(nc));
    if constexpr (GAMMA) {
      uint32_t sq;
      asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(sq) : "r"(v), "r"(v));
      asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(acc) : "r"(sq), "r"(G2b[j]), "r"(acc));
    } else {
      asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(acc) : "r"(v), "r"(v), "r"(acc));
    }
  }
  return __fadd_rn(bits_f32(acc << 16), bits_f32(acc & 0xffff0000u));
}

// The same sum in fp32 from the signed pairs t2 (f16 inputs).
template <bool GAMMA>
__device__ __forceinline__ float clip_excess_f32(const unsigned long long (&t2)[16], float c, const float* Gw) {
  const unsigned long long C2 = pack2(c, c);
  unsigned long long acc = 0ull;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const f2 v = unpack2(add2(t2[j] | 0x8000000080000000ull, C2));  // c - |t|: negative where clipped
    const unsigned long long vv = pack2(fminf(v.x, 0.0f), fminf(v.y, 0.0f));
    if constexpr (GAMMA) {
      acc = fma2(mul2(vv, vv), load_g2(Gw, j), acc);
    } else {
      acc = fma2(vv, vv, acc);
    }
  }
  const f2 r = unpack2(acc);
  return __fadd_rn(r.x, r.y);
}

// gamma^2 pairs 4q .. 4q+3 of the warp's block column (two broadcast loads).
__device__ __forceinline__ void load_g2_quad(const float* Gw, int q, unsigned long long (&g)[4]) {
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(g[0]), "=l"(g[1]) : "r"(smem_u32(Gw + 8 * q)));
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(g[2]), "=l"(g[3]) : "r"(smem_u32(Gw + 8 * q + 4)));
}

// E2M1 round trip of four signed pairs: the values as f16x2 words and the
// four code bytes packed into one word (pair k in byte k, element 2j in the
// low nibble of its byte).
__device__ __forceinline__ uint32_t e2m1_quad(const unsigned long long (&x)[4], uint32_t (&h)[4]) {
  const f2 a = unpack2(x[0]), b = unpack2(x[1]), c = unpack2(x[2]), d = unpack2(x[3]);
  uint32_t codes;
  asm("{\n\t.reg .b8 t0, t1, t2, t3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t0, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t1, %8, %7;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t2, %10, %9;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t3, %12, %11;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, t0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, t1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, t2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, t3;\n\t"
      "mov.b32 %4, {t0, t1, t2, t3};\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3]), "=r"(codes)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y), "f"(d.x), "f"(d.y));
  return codes;
}

// fl(q * s + t) per element for q an f16 pair (E2M1 values), s an f16 scale
// (a power of two) and t an fp32 pair: one mixed-precision FMA per element,
// rounded once like the fp32 form (the product of two f16 values is exact).
__device__ __forceinline__ float fma_f16_f32(uint16_t q, uint16_t s, float t) {
  float r;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(r) : "h"(q), "h"(s), "f"(t));
  return r;
}

__device__ __forceinline__ unsigned long long fma2_f16(uint32_t q2, uint16_t s, unsigned long long t) {
  const f2 tt = unpack2(t);
  return pack2(fma_f16_f32(static_cast<uint16_t>(q2 & 0xffffu), s, tt.x),
               fma_f16_f32(static_cast<uint16_t>(q2 >> 16), s, tt.y));
}

__device__ __forceinline__ unsigned long long f16x2_to_f32x2(uint32_t h) {
  const __half2 hh = *reinterpret_cast<const __half2*>(&h);
  return pack2(__low2float(hh), __high2float(hh));
}

// Errors of candidates f and f+1 in one pass over the block's signed pairs,
// with each candidate's packed codes.  Per element and candidate, in the
// reference's rounding: x = t / 2^e (exact here: |t| >= 2^-133 and e <= 15,
// so nothing underflows; +0 is added to turn -0 into +0 as the reference's
// sign rule does), q = E2M1(x) by hardware RNE with saturation,
// dW = fl(q*2^e - t) (computed as fl(t - q*2^e), the same magnitude, by one
// mixed-precision FMA per element on q's f16 value),
// fl(dW^2), fl(. * gamma^2), then the lane partials and their left-to-right
// sum, / 32.  The codes of x are the final encode's codes when e wins
// (core.py:242-249 recomputes the same x).
template <bool GAMMA>
__device__ __forceinline__ void two_candidate_errors(const unsigned long long (&t2)[16], int f, const float* Gw,
                                                     const QuantParams& P, float& e0, float& e1, uint4& pk0,
                                                     uint4& pk1) {
  const unsigned long long Z2 = pack2(P.zero, P.zero);
  const unsigned long long NZ2 = pack2(P.negzero, P.negzero);
  const float i0 = exp2i(-f), s0 = -exp2i(f);
  const unsigned long long I0 = pack2(i0, i0), I1 = pack2(0.5f * i0, 0.5f * i0);
  // -2^f and -2^(f+1) as f16 (exact: here -23 <= f <= 14) for the mixed-precision
  // t - q * 2^e, one FMA per element instead of a conversion plus half an FFMA2.
  const uint16_t hs0 = __half_as_ushort(__float2half_rn(s0)), hs1 = __half_as_ushort(__float2half_rn(2.0f * s0));
  unsigned long long p0[4], p1[4];
  uint32_t w0[4], w1[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    unsigned long long xa[4], xb[4], g[4];
    uint32_t ha[4], hb[4];
    if constexpr (GAMMA) load_g2_quad(Gw, q, g);  // issued early: its latency hides behind the conversions
#pragma unroll
    for (int lp = 0; lp < 4; ++lp) {
      xa[lp] = fma2(t2[q * 4 + lp], I0, Z2);
      xb[lp] = fma2(t2[q * 4 + lp], I1, Z2);
    }
    w0[q] = e2m1_quad(xa, ha);
    w1[q] = e2m1_quad(xb, hb);
#pragma unroll
    for (int lp = 0; lp < 4; ++lp) {
      const int j = q * 4 + lp;
      const unsigned long long da = fma2_f16(ha[lp], hs0, t2[j]);
      const unsigned long long db = fma2_f16(hb[lp], hs1, t2[j]);
      unsigned long long sa = mul2_rounded(da, da, NZ2);
      unsigned long long sb = mul2_rounded(db, db, NZ2);
      if constexpr (GAMMA) {
        sa = mul2_rounded(sa, g[lp], NZ2);
        sb = mul2_rounded(sb, g[lp], NZ2);
      }
      p0[lp] = (q == 0) ? sa : add2(p0[lp], sa);
      p1[lp] = (q == 0) ? sb : add2(p1[lp], sb);
    }
  }
  float a0 = __fadd_rn(unpack2(p0[0]).x, unpack2(p0[0]).y);
  float a1 = __fadd_rn(unpack2(p1[0]).x, unpack2(p1[0]).y);
#pragma unroll
  for (int lp = 1; lp < 4; ++lp) {
    a0 = __fadd_rn(__fadd_rn(a0, unpack2(p0[lp]).x), unpack2(p0[lp]).y);
    a1 = __fadd_rn(__fadd_rn(a1, unpack2(p1[lp]).x), unpack2(p1[lp]).y);
  }
  e0 = __fmul_rn(a0, 0.03125f);
  e1 = __fmul_rn(a1, 0.03125f);
  pk0 = make_uint4(w0[0], w0[1], w0[2], w0[3]);
  pk1 = make_uint4(w1[0], w1[1], w1[2], w1[3]);
}

// Error of one candidate e from the signed pairs: the arithmetic of
// two_candidate_errors without the codes.  t / 2^e is exact for the exponents
// the fast path evaluates here (f - 8 <= e <= f + 2 <= 16).
template <bool GAMMA>
__device__ __forceinline__ float one_candidate_error(const unsigned long long (&t2)[16], int e, const float* Gw,
                                                     const QuantParams& P) {
  const unsigned long long Z2 = pack2(P.zero, P.zero);
  const unsigned long long NZ2 = pack2(P.negzero, P.negzero);
  const float i = exp2i(-e), sc = -exp2i(e);
  const unsigned long long I2 = pack2(i, i), S2 = pack2(sc, sc);
  unsigned long long p[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int lp = 0; lp < 4; ++lp) {
      const int j = q * 4 + lp;
      const f2 x = unpack2(fma2(t2[j], I2, Z2));
      uint32_t h2;
      asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
          : "=r"(h2) : "f"(x.y), "f"(x.x));
      const unsigned long long d = fma2(f16x2_to_f32x2(h2), S2, t2[j]);
      unsigned long long sq = mul2_rounded(d, d, NZ2);
      if constexpr (GAMMA) sq = mul2_rounded(sq, load_g2(Gw, j), NZ2);
      p[lp] = (q == 0) ? sq : add2(p[lp], sq);
    }
  }
  float acc = __fadd_rn(unpack2(p[0]).x, unpack2(p[0]).y);
#pragma unroll
  for (int lp = 1; lp < 4; ++lp) acc = __fadd_rn(__fadd_rn(acc, unpack2(p[lp]).x), unpack2(p[lp]).y);
  return __fmul_rn(acc, 0.03125f);
}

// Error of candidate e for the block of lane `src`, by the whole warp: lane l
// takes element l (staged through the warp's 32-float scratch `Xw`) and forms
// fl(fl(t - q*2^e)^2 [* gamma^2]) as one_candidate_error does; the lane
// partials ((x_l + x_{l+8}) + x_{l+16}) + x_{l+24} and their left-to-right sum
// are the reference's 8-lane order.  Warp-collective; every lane gets the error.
template <bool GAMMA>
__device__ __forceinline__ float warp_candidate_error(const unsigned long long (&t2)[16], int e, int src, int lane,
                                                      const float* Gw, float* Xw, const QuantParams& P) {
  __syncwarp();
  if (lane == src) {
#pragma unroll
    for (int j = 0; j < 16; ++j) reinterpret_cast<unsigned long long*>(Xw)[j] = t2[j];
  }
  __syncwarp();
  const float t = Xw[lane];
  const float x = __fmaf_rn(t, exp2i(-e), P.zero);
  uint32_t h2;
  asm("{\n\t.reg .b8 c;\n\tcvt.rn.satfinite.e2m1x2.f32 c, %1, %2;\n\tcvt.rn.f16x2.e2m1x2 %0, c;\n\t}"
      : "=r"(h2) : "f"(0.0f), "f"(x));
  const float q = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xffffu)));
  const float d = __fmaf_rn(q, -exp2i(e), t);
  float sq = __fmul_rn(d, d);
  if constexpr (GAMMA) sq = __fmul_rn(sq, Gw[lane]);
  float part = __fadd_rn(sq, __shfl_down_sync(0xffffffffu, sq, 8));
  part = __fadd_rn(part, __shfl_down_sync(0xffffffffu, sq, 16));
  part = __fadd_rn(part, __shfl_down_sync(0xffffffffu, sq, 24));
  float acc = __shfl_sync(0xffffffffu, part, 0);
#pragma unroll
  for (int l = 1; l < 8; ++l) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, part, l));
  __syncwarp();  // Xw is reused by the next block
  return __fmul_rn(acc, 0.03125f);
}

// Warp-collective (the extra candidates run under warp votes): every lane
// calls it; `active` marks lanes whose tile row exists.  Reads its block (tile
// row `lane`, block column w) from the stage; lane 0 releases the stage on
// `release` once the warp has read it.  Returns the E8M0 byte (or
// kRareBlock) and the packed codes; `nonfinite` reports NaN/inf.
template <int DT, int OBJ, int QM>
__device__ __forceinline__ uint32_t quantize_block_fast(bool active, const QuantParams& P, const uint8_t* stage,
                                                        int w, int lane, const float* Gw, float* Xw, const uint32_t* G2b,
                                                        uint64_t* release, uint4& packed, bool& nonfinite) {
  constexpr bool GAMMA = OBJ == kObjGamma;
  float amax, second;
  unsigned long long t2[16];
  {
    uint32_t words[16];
    stage_words(stage, w, lane, words);
    // Magnitude order statistics on the raw 16-bit patterns (sign-magnitude:
    // the integer order is the order of |value|; NaN/inf on top).
    uint32_t m1 = 0, m2 = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t a = words[k] & 0x7fff7fffu;
      if constexpr (QM == kQTop2) m2 = __vmaxu2(m2, __vminu2(m1, a));
      m1 = __vmaxu2(m1, a);
      t2[k] = word_pair<DT>(words[k]);
    }
    const uint32_t lo1 = m1 & 0xffffu, hi1 = m1 >> 16;
    const uint32_t top1 = max(lo1, hi1);
    uint32_t top2 = 0;
    if constexpr (QM == kQTop2) top2 = max(min(lo1, hi1), max(m2 & 0xffffu, m2 >> 16));
    if constexpr (DT == MXW_BF16) {
      nonfinite = top1 >= 0x7f80u;
      amax = bits_f32(top1 << 16);
      second = bits_f32(top2 << 16);
    } else {
      nonfinite = top1 >= 0x7c00u;
      amax = __half2float(__ushort_as_half(static_cast<unsigned short>(top1)));
      second = __half2float(__ushort_as_half(static_cast<unsigned short>(top2)));
    }
  }
  // Release the stage only once every lane's loads have returned: the arrive
  // waits on a warp reduction of the statistics computed from them.
  const uint32_t loaded = __reduce_or_sync(0xffffffffu, f32_bits(amax));  // sign clear: never all ones
  if (lane == 0 && loaded != 0xffffffffu) mbar_arrive(release);
  unsigned long long unused_nt2[16];
  const float anchor = fmaxf(block_anchor<QM>(amax, second, unused_nt2, P), 1e-6f);
  const bool near_zero = amax < 1e-6f;
  bool fast = active && !near_zero && !nonfinite;
  const int f = fast ? floor_log2_div6(anchor) : 0;
  const int safe_e = fast ? ceil_log2_div6(fmaxf(amax, 1e-12f)) : 0;
  // f >= -23 (the anchor is at least 1e-6), so f - depth is never clamped;
  // f <= 14 keeps t / 2^e exact for the codes of f and f+1.
  fast = fast && f <= 14 && safe_e <= f + 2;

  float e_f, e_f1;
  uint4 pk_f, pk_f1;
  two_candidate_errors<GAMMA>(t2, f, Gw, P, e_f, e_f1, pk_f, pk_f1);
  fast = fast && !isnan(e_f) && !isnan(e_f1);
  const float e_hi = fminf(e_f, e_f1);

  // Clipping candidates below f: certified losers, or evaluated below.
  bool need_low = fast && P.depth > 0;
  if (__any_sync(0xffffffffu, need_low)) {
    const float c = __fmul_rn(exp2i(f), 3.0f);  // 6 * 2^(f-1), exact
    if constexpr (!GAMMA) {
      const float v1 = fmaxf(__fsub_rn(amax, c), 0.0f);
      const float v2 = QM == kQTop2 ? fmaxf(__fsub_rn(second, c), 0.0f) : 0.0f;
      const float lb = __fmul_rn(__fadd_rn(__fmul_rn(v1, v1), __fmul_rn(v2, v2)), 0.03125f);
      need_low = need_low && !lb_prunes(lb, e_hi);
    }
    if (__any_sync(0xffffffffu, need_low)) {
      float sum;
      if constexpr (DT == MXW_BF16) {
        uint32_t wd[16];  // the bf16 words again, from the exact fp32 pairs
#pragma unroll
        for (int j = 0; j < 16; ++j)
          wd[j] = __byte_perm(static_cast<uint32_t>(t2[j]), static_cast<uint32_t>(t2[j] >> 32), 0x7632);
        sum = clip_excess_bf16<GAMMA>(wd, c, G2b);
      } else {
        sum = clip_excess_f32<GAMMA>(t2, c, Gw);
      }
      need_low = need_low && !lb_prunes(__fmul_rn(sum, 0.03125f), e_hi);
    }
  }
  const bool need_safe = fast && safe_e == f + 2;
  const int lo_e = f - P.depth;

  // Argmin in the reference's order (core.py:220-238): strict <, the first
  // candidate is the initial choice, NaN propagates through the minimum.
  int raw = lo_e;
  float best = __int_as_float(0x7f800000);
  if (__any_sync(0xffffffffu, need_low)) {
    for (int k = 0; k < P.depth; ++k) {
      const float err = one_candidate_error<GAMMA>(t2, lo_e + k, Gw, P);
      if (need_low) {
        if (err < best) raw = lo_e + k;
        best = nan_min(best, err);
      }
    }
  }
  if (e_f < best) raw = f;
  best = nan_min(best, e_f);
  if (e_f1 < best) raw = f + 1;
  best = nan_min(best, e_f1);
  bool run_safe = need_safe;
  if (!GAMMA && __any_sync(0xffffffffu, run_safe)) {
    // Unweighted objective only.  The safe candidate (f+2) comes last, so it
    // wins only with an error strictly below `best`.  Every E2M1 value at
    // scale f+2 is a multiple of 2^(f+1), so each element's error is at least
    // its distance to that lattice: (2^(f+1) * |v - rint(v)|)^2 with
    // v = t / 2^(f+1) (rint by the 1.5 * 2^23 add, exact for |v| <= 12 here).
    // Measured: a 2 % gain unweighted; with gamma weights the extra loads cost
    // more than it saves, so weighted blocks skip the bound.
    const float iv = exp2i(-(f + 1));
    const unsigned long long IV = pack2(iv, iv), M2 = pack2(12582912.0f, 12582912.0f);
    const unsigned long long NM2 = pack2(-12582912.0f, -12582912.0f), NEG2 = pack2(-1.0f, -1.0f);
    unsigned long long acc = 0ull;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const unsigned long long v = mul2(t2[j], IV);
      const unsigned long long r = fma2(add2(add2(v, M2), NM2), NEG2, v);  // v - rint(v)
      acc = fma2(r, r, acc);
    }
    const f2 a2 = unpack2(acc);
    const float lb = __fmul_rn(__fmul_rn(__fadd_rn(a2.x, a2.y), exp2i(2 * f + 2)), 0.03125f);
    run_safe = run_safe && !lb_prunes(lb, best);
  }
  // The safe candidate is needed by a few scattered blocks (about 2 % with
  // gamma weights, but then in half of the warps): each such block is
  // evaluated by the whole warp, lane = element, instead of by its thread
  // with the other 31 lanes idle.
  uint32_t need = __ballot_sync(0xffffffffu, run_safe);
  while (need) {
    const int src = __ffs(need) - 1;
    need &= need - 1;
    const float err = warp_candidate_error<GAMMA>(t2, __shfl_sync(0xffffffffu, safe_e, src), src, lane, Gw, Xw, P);
    if (lane == src && err < best) raw = safe_e;
  }

  if (near_zero && active && !nonfinite) {
    // t is replaced by zeros (core.py:194-195): the first candidate wins,
    // with f from the clamped anchor 1e-6.
    packed = make_uint4(0u, 0u, 0u, 0u);
    return static_cast<uint32_t>(floor_log2_div6(anchor) - P.depth + 127);
  }
  if (!fast) return kRareBlock;
  if (raw == f) {
    packed = pk_f;
  } else if (raw == f + 1) {
    packed = pk_f1;
  } else {
    encode_pairs([&](int j) { return t2[j]; }, P, raw, packed);  // an extra candidate won
  }
  return static_cast<uint32_t>(raw + 127);
}

// --------------------------------------------------------------- TMA kernel

// (strip, row tile) of consecutive strip-major tiles: one 64-bit division per
// CTA instead of one per tile.
struct TileCursor {
  int64_t strip, rt;
  __device__ __forceinline__ TileCursor(int64_t t, int64_t n_row_tiles) : strip(t / n_row_tiles), rt(t % n_row_tiles) {}
  __device__ __forceinline__ void advance(int64_t n_row_tiles) {
    if (++rt == n_row_tiles) {
      rt = 0;
      ++strip;
    }
  }
};

template <int DT, int OBJ, int QM>
__global__ void __launch_bounds__(kQuantThreads, (OBJ == kObjHess || DT == MXW_F32) ? 1 : 2)
    quantize_tma_kernel(const __grid_constant__ CUtensorMap map, const __grid_constant__ CUtensorMap out_map,
                        const QuantParams P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  constexpr int kStageBytes = Elem<DT>::kStageBytes;
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint8_t* stages = smem;
  uint8_t* out_stage = smem + kStages * kStageBytes;               // [ring][32 rows][128 B], 128B-swizzled
  uint8_t* scale_stage = out_stage + kOutBuffers * kOutTileBytes;  // [ring][32 rows][8 B]
  float* Hs = reinterpret_cast<float*>(scale_stage + kOutBuffers * kScaleTileBytes);
  float* Gs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(Hs) + (OBJ == kObjHess ? kTileBlocks * 1024 * 4 : 0));
  // One block's 32 elements per consumer warp, for the warp-cooperative candidate evaluation.
  float* Xs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(Gs) + (OBJ == kObjGamma ? kTileBlocks * kGammaWords * 4 : 0));
  uint64_t* full = reinterpret_cast<uint64_t*>(Xs + kTileBlocks * kBlock);
  uint64_t* empty = full + kStages;
  uint64_t* out_full = empty + kStages;
  uint64_t* out_empty = out_full + kOutBuffers;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // This CTA's contiguous range of tiles, strip-major.
  const int64_t t_begin = P.n_tiles * blockIdx.x / gridDim.x;
  const int64_t t_end = P.n_tiles * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int i = 0; i < kOutBuffers; ++i) {
      mbar_init(&out_full[i], kConsumerWarps);
      mbar_init(&out_empty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kStoreWarp) {
    // ---------------- store warp: one TMA store + 32 scale rows per tile.
    bool ok = true;
    int64_t it = 0;
    const bool scale_words = (P.nb % 8 == 0) && (reinterpret_cast<uintptr_t>(P.scales) % 8 == 0);
    TileCursor cur(t_begin, P.n_row_tiles);
    for (int64_t t = t_begin; t < t_end; ++t, ++it, cur.advance(P.n_row_tiles)) {
      const int64_t strip = cur.strip, rt = cur.rt;
      const int buf = static_cast<int>(it % kOutBuffers);
      if (!__all_sync(0xffffffffu, mbar_wait(&out_full[buf], static_cast<uint32_t>((it / kOutBuffers) & 1)))) {
        ok = false;
        break;
      }
      if (lane == 0) {
        tma_store_2d(&out_map, out_stage + buf * kOutTileBytes, static_cast<int32_t>(strip * kTileBlocks * 16),
                     static_cast<int32_t>(rt * kTileRows));
        bulk_commit_group();
      }
      const uint8_t* sstage = scale_stage + buf * kScaleTileBytes;
      const int64_t r = rt * kTileRows + lane;
      const int64_t b0 = strip * kTileBlocks;
      if (r < P.rows) {
        if (scale_words && b0 + kTileBlocks <= P.nb) {
          *reinterpret_cast<uint2*>(P.scales + r * P.nb + b0) = *reinterpret_cast<const uint2*>(sstage + lane * kTileBlocks);
        } else {
          for (int k = 0; k < kTileBlocks && b0 + k < P.nb; ++k) P.scales[r * P.nb + b0 + k] = sstage[lane * kTileBlocks + k];
        }
      }
      __syncwarp();
      // Release the buffer stored kOutBuffers-1 tiles ago: at most
      // kOutBuffers-1 stores may still read shared memory.
      if (lane == 0) {
        bulk_wait_group_read<kOutBuffers - 1>();
        if (it >= kOutBuffers - 1) mbar_arrive(&out_empty[(it - (kOutBuffers - 1)) % kOutBuffers]);
      }
    }
    if (lane == 0) {
      bulk_wait_group_all();
      if (!ok && P.flags) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
    }
    return;
  }

  if (warp == kProducerWarp) {
    // ---------------- producer warp: one elected lane issues all TMA loads.
    if (lane == 0) {
      prefetch_tensormap(&map);
      int64_t issued = 0;
      bool ok = true;
      TileCursor cur(t_begin, P.n_row_tiles);
      for (int64_t t = t_begin; t < t_end; ++t, ++issued, cur.advance(P.n_row_tiles)) {
        const int64_t strip = cur.strip, rt = cur.rt;
        const int64_t col0 = strip * kTileBlocks * kBlock;
        const int64_t left = (P.cols - col0 + Elem<DT>::kBoxCols - 1) / Elem<DT>::kBoxCols;
        const int boxes = left < Elem<DT>::kBoxesPerStage ? static_cast<int>(left) : Elem<DT>::kBoxesPerStage;
        const int s = static_cast<int>(issued % kStages);
        if (issued >= kStages && !mbar_wait(&empty[s], static_cast<uint32_t>((issued / kStages - 1) & 1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], boxes * kBoxBytes);
        for (int k = 0; k < boxes; ++k)
          tma_load_2d(stages + s * kStageBytes + k * kBoxBytes, &map, &full[s],
                      static_cast<int32_t>(col0 + k * Elem<DT>::kBoxCols), static_cast<int32_t>(rt * kTileRows));
      }
      // Never leave with copies in flight: wait for the last issued stages.
      for (int64_t i = (issued > kStages ? issued - kStages : 0); i < issued; ++i) {
        if (!mbar_wait(&full[i % kStages], static_cast<uint32_t>((i / kStages) & 1))) ok = false;
      }
      if (!ok && P.flags) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
    }
    return;
  }

  // ---------------- consumer warps: warp w owns block column strip*8 + w.
  unsigned long long g2[16];  // unused here: gamma^2 lives in shared memory (Gw)
  float* Hw = Hs + warp * 1024;
  float* Gw = Gs + warp * kGammaWords;
  int64_t cur_strip = -1;
  bool valid_col = false;
  int64_t b = 0;
  bool any_nonfinite = false;
  bool any_rare = false;  // a block marked kRareBlock: the rare-block pass has work
  int64_t it = 0;
  TileCursor cur(t_begin, P.n_row_tiles);
  for (int64_t t = t_begin; t < t_end; ++t, ++it, cur.advance(P.n_row_tiles)) {
    const int64_t strip = cur.strip, rt = cur.rt;
    if (strip != cur_strip) {
      cur_strip = strip;
      b = strip * kTileBlocks + warp;
      valid_col = b < P.nb;
      if (valid_col) load_column_state<OBJ>(P, b, lane, Hw, Gw);
    }
    const int s = static_cast<int>(it % kStages);
    // Warp-uniform verdict: a lane that timed out takes the whole warp out.
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>((it / kStages) & 1)))) {
      if (P.flags && lane == 0) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
      break;
    }
    const int buf = static_cast<int>(it % kOutBuffers);
    uint8_t* ostage = out_stage + buf * kOutTileBytes;
    uint8_t* sstage = scale_stage + buf * kScaleTileBytes;
    uint4 pk = make_uint4(0u, 0u, 0u, 0u);
    uint32_t sc = 0;
    if (valid_col) {
      const bool active = rt * kTileRows + lane < P.rows;
      if constexpr (FastPath<DT, OBJ, QM>::value) {
        // Warp-collective; the stage stays held until its warp evaluation is done.
        // Warp-collective; it releases the stage once the warp has read it.
        bool nf = false;
        sc = quantize_block_fast<DT, OBJ, QM>(active, P, stages + s * kStageBytes, warp, lane, Gw, Xs + warp * kBlock,
                                              reinterpret_cast<const uint32_t*>(Gw + kBlock), &empty[s], pk, nf);
        any_nonfinite |= active && nf;
      } else {
        BlockData<DT> B;
        read_block_smem<DT, QM>(stages + s * kStageBytes, warp, lane, B);
        const uint32_t loaded = __reduce_or_sync(0xffffffffu, f32_bits(B.amax));  // as in quantize_block_fast
        if (lane == 0 && loaded != 0xffffffffu) mbar_arrive(&empty[s]);
        if (active) {
          any_nonfinite |= B.nonfinite;
          sc = quantize_one_block<DT, OBJ, QM, true, true, OBJ != kObjHess>(B, P, g2, Hw, pk, Gw);
        }
      }
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // Stage: row `lane`, 16-byte chunk `warp`, 128B-swizzled (chunk ^ row%8)
    // to match the output tensor map.  Wait for the buffer to be free first.
    if (it >= kOutBuffers &&
        !__all_sync(0xffffffffu, mbar_wait(&out_empty[buf], static_cast<uint32_t>((it / kOutBuffers - 1) & 1)))) {
      if (P.flags && lane == 0) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
      break;
    }
    *reinterpret_cast<uint4*>(ostage + lane * 128 + ((warp ^ (lane & 7)) << 4)) = pk;
    sstage[lane * kTileBlocks + warp] = static_cast<uint8_t>(sc);
    any_rare |= valid_col && rt * kTileRows + lane < P.rows && sc == kRareBlock;
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&out_full[buf]);
  }
  if (P.flags && __any_sync(0xffffffffu, any_nonfinite) && lane == 0) atomicOr(P.flags, MXW_FLAG_NONFINITE);
  if (P.flags && __any_sync(0xffffffffu, any_rare) && lane == 0) atomicOr(P.flags, MXW_FLAG_RARE);
}

// ------------------------------------------------------ rare-block fixup

// One block read from global memory as fp32 (exact for every input type) and
// quantized with both error forms available (see quantize_one_block).
template <int DT, int OBJ, int QM>
__device__ __forceinline__ uint32_t quantize_block_slow(const QuantParams& P, int64_t row, int64_t blk, uint4* packed) {
  BlockData<MXW_F32> B;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int64_t i = row * P.ld + blk * kBlock + 2 * j;
    float x0, x1;
    if constexpr (DT == MXW_BF16) {
      const uint16_t* p = static_cast<const uint16_t*>(P.weight) + i;
      x0 = bits_f32(static_cast<uint32_t>(p[0]) << 16);
      x1 = bits_f32(static_cast<uint32_t>(p[1]) << 16);
    } else if constexpr (DT == MXW_F16) {
      const __half* p = static_cast<const __half*>(P.weight) + i;
      x0 = __half2float(p[0]);
      x1 = __half2float(p[1]);
    } else {
      const float* p = static_cast<const float*>(P.weight) + i;
      x0 = p[0];
      x1 = p[1];
    }
    B.t2[j] = pack2(x0, x1);
  }
  finish_stats_f32<MXW_F32, QM>(B, B.t2);
  unsigned long long g2[16];
  if constexpr (OBJ == kObjGamma) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float ga = P.gamma[blk * kBlock + 2 * j], gb = P.gamma[blk * kBlock + 2 * j + 1];
      g2[j] = pack2(__fmul_rn(ga, ga), __fmul_rn(gb, gb));
    }
  }
  uint4 pk;
  const float* Hb = OBJ == kObjHess ? P.hessian + blk * 1024 : nullptr;
  const uint32_t sc = quantize_one_block<MXW_F32, OBJ, QM, false>(B, P, g2, Hb, pk);
  *packed = pk;
  return sc;
}

// Runs after quantize_tma_kernel (unweighted / gamma objectives, same stream):
// finds the blocks it marked kRareBlock and quantizes them in full.  One wave
// of threads reads the scale bytes once (1 byte per 32 weights) in 16-byte
// chunks, four independent loads in flight per thread; marked blocks are rare.
constexpr int kFixupChunk = 16;

template <int DT, int OBJ, int QM>
__device__ __forceinline__ void fixup_block(const QuantParams& P, int64_t idx) {
  const int64_t r = idx / P.nb, b = idx % P.nb;
  uint4 pk;
  const uint32_t sc = quantize_block_slow<DT, OBJ, QM>(P, r, b, &pk);
  *reinterpret_cast<uint4*>(P.packed + r * (P.cols / 2) + b * 16) = pk;
  P.scales[idx] = static_cast<uint8_t>(sc);
}

template <int DT, int OBJ, int QM>
__global__ void __launch_bounds__(256) quantize_fixup_kernel(const QuantParams P, const uint32_t gate) {
  // With a flag word, the earlier passes reported whether any block can be
  // marked: MXW_FLAG_RARE after the main pass, MXW_FLAG_NONFINITE after the
  // block-Hessian exact pass (which leaves only non-finite blocks marked).
  if (P.flags && (*reinterpret_cast<volatile const uint32_t*>(P.flags) & gate) == 0) return;
  const int64_t total = P.rows * P.nb;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (reinterpret_cast<uintptr_t>(P.scales) % 16 == 0) {
    const int64_t chunks = total / kFixupChunk;
    for (int64_t c0 = tid; c0 < chunks; c0 += 4 * stride) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t c = c0 + u * stride;
        v[u] = c < chunks ? *reinterpret_cast<const uint4*>(P.scales + c * kFixupChunk) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t m = __vcmpeq4(w[q], 0xffffffffu);  // 0xff per marked byte
          if (m) {
            for (int k = 0; k < 4; ++k)
              if ((m >> (8 * k)) & 1u) fixup_block<DT, OBJ, QM>(P, (c0 + u * stride) * kFixupChunk + 4 * q + k);
          }
        }
      }
    }
    // The tail beyond the last whole chunk.
    for (int64_t i = chunks * kFixupChunk + tid; i < total; i += stride)
      if (P.scales[i] == kRareBlock) fixup_block<DT, OBJ, QM>(P, i);
  } else {
    for (int64_t i = tid; i < total; i += stride)
      if (P.scales[i] == kRareBlock) fixup_block<DT, OBJ, QM>(P, i);
  }
}

// ------------------------------ block-Hessian objective: tensor-core screening
//
// The block-Hessian error of a candidate exponent e is E = D^T H D over the
// block's 32 elements, D = q(t / 2^e) * 2^e - t, H the block's 32x32 Hessian
// (core.py:227-229).  The reference rounds it in a fixed order: per output d
// an fp32 FMA chain over s, then the products summed in 8-lane order.  Doing
// that on CUDA cores costs 1,024 FMA per block and candidate, reading H from
// shared memory for each.  Here the tensor cores screen instead:
//
//   * the screening works on D / 2^e = q(x) - x (x = t / 2^e): the form
//     scales exactly by 2^(2e).  It is exact in bf16 when |x| < 512 (at most
//     8 significant bits: t has 8 and q - x is a multiple of x's last place
//     no larger than |x|), and H = Hh + Hl in two bf16 halves to 2^-16
//     relative;
//   * per tile of 128 rows x 2 block columns, each thread writes its block's
//     D / 2^e for up to 4 candidates into shared memory (K-major, no
//     swizzle), and one thread issues tcgen05.mma (M = 128 rows, N = 32,
//     K = 32, both H halves) into TMEM: W = D * H for every row at once;
//   * each thread reads its row of W back (tcgen05.ld) and forms
//     E' = sum_d W_d D_d in packed fp32 pairs, with a bound
//     |E' - E_reference| <= 4e-5 * A where
//     A >= sum_{s,d} |D_s| |H_sd| |D_d| (2^-16 from the split, 2^-17 from the
//     tensor core's fp32 accumulation, about 46 fp32 roundings on each side);
//     A is (sum_s |D_s| sqrt(H_ss))^2 when every |H_sd| <= sqrt(H_ss H_dd)
//     (checked per block column), else max|D| * sum_s |D_s| sum_d |H_sd|;
//   * the candidate with the least E' (earliest on ties) is the reference's
//     choice when every other candidate's E' exceeds it by more than both
//     bounds; otherwise the block gets the rare marker and
//     quantize_fixup_hess_kernel evaluates it exactly, one warp per block
//     (blocks with non-finite elements: quantize_fixup_kernel, one thread).
//
// Candidates follow the reference's order (core.py:201-209): f - depth ..
// f + 1, then the no-clipping exponent when it is f + 2.  Blocks outside
// that domain (non-finite, block scales of 2^15 and above, safe >= f + 3) also
// take the exact pass.  Rounds of 4 candidates keep TMEM at 256 columns, so
// two CTAs share an SM and one computes while the other waits for its MMAs.

constexpr int kHtRows = 128;                              // weight rows per tile (TMEM lanes)
constexpr int kHtCols = 2;                                // block columns per tile
constexpr int kHtStages = 2;
constexpr int kHtStageBytes = kHtRows * 128;              // 128 rows x 64 two-byte elements
constexpr int kHtRound = 2;                               // candidates per MMA round
constexpr int kHtBufs = 2;                                // rounds in flight (D and TMEM buffers)
constexpr int kHtDBytes = kHtRows * 64;                   // bf16 D of one candidate and block column
constexpr int kHtHBytes = 32 * 64;                        // one bf16 half of a 32x32 block Hessian
constexpr uint32_t kHtTmemCols = kHtBufs * kHtRound * kHtCols * 32;  // 256
constexpr uint32_t kHtTmemBuf = kHtRound * kHtCols * 32;
constexpr int kHtConsumerWarps = 8;
constexpr int kHtProducerWarp = 8;
constexpr int kHtMmaWarp = 9;
constexpr int kHtThreads = 10 * 32;
constexpr float kHtTol = 4e-5f;
constexpr float kHtTolInexact = 4e-5f + 0.0079f;  // plus (2 * 2^-8 + 2^-16) x 1.01 for a rounded D
// Shared memory: stages | D [round][col] | H halves [col][hi, lo] | per-column
// bound data (sqrt(H_ss) and sum_d |H_sd|, 32 each, then the CS flag) | barriers.
constexpr int kHtOffD = kHtStages * kHtStageBytes;
constexpr int kHtDBuf = kHtRound * kHtCols * kHtDBytes;    // one round's D
constexpr int kHtOffH = kHtOffD + kHtBufs * kHtDBuf;
constexpr int kHtOffB = kHtOffH + kHtCols * 2 * kHtHBytes;
constexpr int kHtOffBar = kHtOffB + kHtCols * 68 * 4;
// Output hand-off slots [quarter][lane]: 16 packed bytes, then the scale byte (after the barriers
// and the TMEM slot).
constexpr int kHtOffPair = (kHtOffBar + (2 * kHtStages + 2 * kHtBufs + 9) * 8 + 16 + 15) & ~15;
constexpr size_t kHtSmem = 1024 + kHtOffPair + 4 * 32 * 16 + 4 * 32 * 4;

// Byte offset of row r's 16-byte chunk kc (elements 8kc .. 8kc+7) in a K-major
// no-swizzle operand of K = 32: 8-row x 16-byte core matrices, 128 bytes
// apart along K and 512 bytes apart along M.
__device__ __forceinline__ uint32_t ht_core_offset(int r, int kc) {
  return static_cast<uint32_t>((r >> 3) * 512 + kc * 128 + (r & 7) * 16);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// D / 2^e = q(x) - x with x = t / 2^e, for the block's 16 element pairs, as
// bf16 pairs (exact whenever |x| < 512).  The quadratic form scales exactly
// with 2^(2e), so the screening works on D / 2^e and rescales its result.  Per
// element: x = t * 2^-e from the bf16 word half by one mixed-precision fma
// (exact), E2M1 round trip by hardware RNE, and q - x by one mixed-precision
// subtraction on q's f16 value (exact in fp32).  The sign of a zero is
// irrelevant here: D enters only the quadratic form and its bound.
__device__ __forceinline__ void ht_candidate_d(const uint32_t (&words)[16], int e, uint32_t (&d)[16]) {
  const uint16_t inv = static_cast<uint16_t>(static_cast<uint32_t>(127 - e) << 7);  // bf16 2^-e (|e| < 100 here)
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float x0, x1, d0, d1;
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "fma.rn.f32.bf16 %0, lo, %3, %4;\n\tfma.rn.f32.bf16 %1, hi, %3, %4;\n\t}"
        : "=f"(x0), "=f"(x1) : "r"(words[j]), "h"(inv), "f"(0.0f));
    asm("{\n\t.reg .b8 c;\n\t.reg .b32 h;\n\t.reg .b16 q0, q1;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 c, %3, %2;\n\t"
        "cvt.rn.f16x2.e2m1x2 h, c;\n\t"
        "mov.b32 {q0, q1}, h;\n\t"
        "sub.rn.f32.f16 %0, q0, %2;\n\t"
        "sub.rn.f32.f16 %1, q1, %3;\n\t}"
        : "=f"(d0), "=f"(d1) : "f"(x0), "f"(x1));
    d[j] = bf16x2_rn(d0, d1);
  }
}

__device__ __forceinline__ unsigned long long fma2_rp(unsigned long long a, unsigned long long b,
                                                      unsigned long long c) {
  unsigned long long r;
  asm("fma.rp.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// One candidate's row of the screening, in units of 2^(2e): E' = sum_d W_d D_d
// (W = D H from TMEM, D from its bf16 words in the core layout) and the bound
// A >= sum_{s,d} |D_s| |H_sd| |D_d| on the terms the reference rounds:
// (sum_s |D_s| sqrt(H_ss))^2 when the block column passed the Cauchy-Schwarz
// check (CS), else max|D| * sum_s |D_s| rowsum_s.  Packed pairs: two RN chains
// for E' and two round-up chains for the linear sum.
template <bool CS>
__device__ __forceinline__ void ht_epilogue(const float (&w)[32], uint32_t src, int r_tile, const float* cb,
                                            float& e_out, float& a_out) {
  unsigned long long ea = 0ull, eb = 0ull, aa = 0ull, ab = 0ull;
  uint32_t dm = 0u;
  const float4* coef = reinterpret_cast<const float4*>(cb + (CS ? 0 : 32));
  // Element pair (s, s + 1) from bf16 word `v`, coefficients (c0, c1).
  auto pair = [&](uint32_t v, int sidx, float c0, float c1, unsigned long long& e, unsigned long long& a) {
    const uint32_t lo = v << 16, hi = v & 0xffff0000u;
    e = fma2(pack2(w[sidx], w[sidx + 1]), pack2(bits_f32(lo), bits_f32(hi)), e);
    a = fma2_rp(pack2(bits_f32(lo & 0x7fffffffu), bits_f32(hi & 0x7fffffffu)), pack2(c0, c1), a);
    if constexpr (!CS) dm = __vmaxu2(dm, v & 0x7fff7fffu);
  };
#pragma unroll
  for (int kc = 0; kc < 4; ++kc) {
    const uint4 v = lds128(src + ht_core_offset(r_tile, kc));
    const float4 c0 = coef[2 * kc], c1 = coef[2 * kc + 1];
    pair(v.x, 8 * kc, c0.x, c0.y, ea, aa);
    pair(v.y, 8 * kc + 2, c0.z, c0.w, eb, ab);
    pair(v.z, 8 * kc + 4, c1.x, c1.y, ea, aa);
    pair(v.w, 8 * kc + 6, c1.z, c1.w, eb, ab);
  }
  const f2 e0 = unpack2(ea), e1 = unpack2(eb), a0 = unpack2(aa), a1 = unpack2(ab);
  e_out = __fadd_rn(__fadd_rn(e0.x, e0.y), __fadd_rn(e1.x, e1.y));
  const float a_lin = __fadd_ru(__fadd_ru(a0.x, a0.y), __fadd_ru(a1.x, a1.y));
  if constexpr (CS) {
    a_out = __fmul_ru(a_lin, a_lin);
  } else {
    const float d_max = bits_f32(max(dm & 0xffffu, dm >> 16) << 16);
    a_out = __fmul_ru(a_lin, d_max);
  }
}

template <int DT, int QM>
__global__ void __launch_bounds__(kHtThreads, 2)
    quantize_hess_tc_kernel(const __grid_constant__ CUtensorMap map, const QuantParams P) {
  static_assert(DT == MXW_BF16, "the screening forms D from bf16 words");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  float* bnd = reinterpret_cast<float*>(smem + kHtOffB);  // [col][68]: sqrt(H_ss) x32, row sums x32, flag
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kHtOffBar);
  uint64_t* empty = full + kHtStages;
  uint64_t* d_ready = empty + kHtStages;    // [kHtBufs]: a round's D is in shared memory
  uint64_t* mma_done = d_ready + kHtBufs;   // [kHtBufs]: a round's products are in TMEM
  uint64_t* strip_bar = mma_done + kHtBufs;  // the consumer warps' barrier around a block-column change
  uint64_t* pair_ready = strip_bar + 1;       // [4]: a column-1 warp's output half is staged
  uint64_t* pair_free = pair_ready + 4;       // [4]: the column-0 warp has taken it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair_free + 4);
  uint4* pair_pk = reinterpret_cast<uint4*>(smem + kHtOffPair);                      // [4][32]
  uint32_t* pair_sc = reinterpret_cast<uint32_t*>(smem + kHtOffPair + 4 * 32 * 16);  // [4][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_strips = (P.nb + kHtCols - 1) / kHtCols;
  const int64_t n_tiles = n_strips * P.n_row_tiles;
  const int64_t t_begin = n_tiles * blockIdx.x / gridDim.x;
  const int64_t t_end = n_tiles * (blockIdx.x + 1) / gridDim.x;
  const int cmax = P.depth + 3;
  const int n_rounds = (cmax + kHtRound - 1) / kHtRound;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kHtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kHtConsumerWarps);
    }
    for (int b = 0; b < kHtBufs; ++b) {
      mbar_init(&d_ready[b], kHtConsumerWarps);
      mbar_init(&mma_done[b], 1);
    }
    mbar_init(strip_bar, kHtConsumerWarps);
    for (int q = 0; q < 4; ++q) {
      mbar_init(&pair_ready[q], 1);
      mbar_init(&pair_free[q], 1);
    }
    fence_mbar_init();
  }
  if (warp == kHtMmaWarp) tmem_alloc(tmem_slot, kHtTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == kHtProducerWarp) {
    if (lane == 0) {
      prefetch_tensormap(&map);
      int64_t i = 0;
      TileCursor cur(t_begin, P.n_row_tiles);
      for (int64_t t = t_begin; t < t_end; ++t, ++i, cur.advance(P.n_row_tiles)) {
        const int s = static_cast<int>(i % kHtStages);
        if (i >= kHtStages && !mbar_wait(&empty[s], static_cast<uint32_t>((i / kHtStages - 1) & 1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kHtStageBytes);
        tma_load_2d(smem + s * kHtStageBytes, &map, &full[s], static_cast<int32_t>(cur.strip * kHtCols * kBlock),
                    static_cast<int32_t>(cur.rt * kHtRows));
      }
      for (int64_t j = (i > kHtStages ? i - kHtStages : 0); j < i; ++j)
        if (!mbar_wait(&full[j % kHtStages], static_cast<uint32_t>((j / kHtStages) & 1))) ok = false;
    }
  } else if (warp == kHtMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32_k(kHtRows, 32);
      // Rounds in order, alternating between the two D / TMEM buffers; round g
      // uses buffer g % 2, whose barriers complete once per use (parity g / 2).
      int64_t round = 0;
      for (int64_t t = t_begin; t < t_end && ok; ++t) {
        for (int r = 0; r < n_rounds; ++r, ++round) {
          const int buf = static_cast<int>(round & 1);
          if (!mbar_wait(&d_ready[buf], static_cast<uint32_t>((round >> 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int cl = 0; cl < kHtRound; ++cl) {
            if (r * kHtRound + cl >= cmax) break;
#pragma unroll
            for (int col = 0; col < kHtCols; ++col) {
              const uint32_t d_tmem = tmem + buf * kHtTmemBuf + static_cast<uint32_t>((cl * kHtCols + col) * 32);
              const uint32_t a = sbase + kHtOffD + buf * kHtDBuf + (cl * kHtCols + col) * kHtDBytes;
              const uint32_t b = sbase + kHtOffH + col * 2 * kHtHBytes;
#pragma unroll
              for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                  const uint64_t ad = make_smem_desc_k_noswz(a + ks * 256, 128, 512);
                  const uint64_t bd = make_smem_desc_k_noswz(b + half * kHtHBytes + ks * 256, 128, 512);
                  mma_bf16_f32(d_tmem, ad, bd, idesc, (ks | half) ? 1u : 0u);
                }
              }
            }
          }
          mma_commit(&mma_done[buf]);
        }
      }
      if (!ok) {
        // Let consumers still waiting on a round see it finish; the timeout flag
        // makes the caller discard the output.
        for (; round < (t_end - t_begin) * n_rounds; ++round) mma_commit(&mma_done[round & 1]);
      }
    }
  } else {
    // ------------------------------------------------- consumers: one block per thread
    const int quarter = warp & 3, col = warp >> 2;
    const int r_tile = quarter * 32 + lane;  // this thread's row of the tile (= TMEM lane)
    const uint32_t my_d = sbase + kHtOffD + col * kHtDBytes;  // + buffer * kHtDBuf + candidate * kHtCols * kHtDBytes
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
    int64_t cur_strip = -1;
    int64_t round = 0;
    int64_t i = 0;
    uint32_t strip_phase = 0;
    // All eight consumer warps meet here; bounded, so a warp that gave up on a
    // wait cannot leave the others blocked.
    auto strip_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(strip_bar);
      const bool met = __all_sync(0xffffffffu, mbar_wait(strip_bar, strip_phase));
      strip_phase ^= 1u;
      return met;
    };
    bool any_nonfinite = false, any_rare = false;
    TileCursor cur(t_begin, P.n_row_tiles);
    for (int64_t t = t_begin; t < t_end; ++t, ++i, cur.advance(P.n_row_tiles)) {
      const int64_t b = cur.strip * kHtCols + col;
      const int64_t row = cur.rt * kHtRows + r_tile;
      const bool valid_col = b < P.nb;
      const bool active = valid_col && row < P.rows;
      const int s = static_cast<int>(i % kHtStages);
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>((i / kHtStages) & 1)))) {
        ok = false;
        break;
      }
      uint32_t words[16];
      {
        const uint8_t* box = smem + s * kHtStageBytes + r_tile * 128;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 v = *reinterpret_cast<const uint4*>(box + (((4 * col + j) ^ (r_tile & 7)) << 4));
          words[4 * j] = v.x;
          words[4 * j + 1] = v.y;
          words[4 * j + 2] = v.z;
          words[4 * j + 3] = v.w;
        }
      }
      // Block statistics (they consume every loaded word) before the stage is
      // released, and the release waits on a warp reduction of them: an
      // mbarrier arrive issued right after the shared-memory loads could
      // complete before their data returns, and the next TMA tile would then
      // overwrite words still in flight.
      uint32_t m1 = 0, m2 = 0;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t a = words[k] & 0x7fff7fffu;
        if constexpr (QM == kQTop2) m2 = __vmaxu2(m2, __vminu2(m1, a));
        m1 = __vmaxu2(m1, a);
      }
      const uint32_t loaded = __reduce_or_sync(0xffffffffu, m1);  // <= 0x7fff7fff
      if (lane == 0 && loaded != 0xffffffffu) mbar_arrive(&empty[s]);
      if (cur.strip != cur_strip) {
        // New block columns: both bf16 halves of H (as the MMA's K-major B
        // operand: row n = d holds H[s][d] over s) and the bound data.  The
        // barrier first: a warp still in the previous tile's epilogue reads
        // the old bound data (the previous tile's MMAs, which read the old
        // halves, have completed: every warp waited for them).
        if (!strip_sync()) {
          ok = false;
          break;
        }
        cur_strip = cur.strip;
        const int idx = r_tile;  // 128 threads per column: row d = idx / 4, chunk kc = idx % 4
        const int d = idx >> 2, kc = idx & 3;
        float hv[8];
        float rowsum = 0.0f;
        bool cs = true;
#pragma unroll
        for (int k = 0; k < 8; ++k) hv[k] = valid_col ? __ldg(P.hessian + b * 1024 + (8 * kc + k) * 32 + d) : 0.0f;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          hi[k] = bf16x2_rn(hv[2 * k], hv[2 * k + 1]);
          const float r0 = __fsub_rn(hv[2 * k], bits_f32(hi[k] << 16));
          const float r1 = __fsub_rn(hv[2 * k + 1], bits_f32(hi[k] & 0xffff0000u));
          lo[k] = bf16x2_rn(r0, r1);
        }
        const uint32_t hb = sbase + kHtOffH + col * 2 * kHtHBytes + ht_core_offset(d, kc);
        sts128(hb, make_uint4(hi[0], hi[1], hi[2], hi[3]));
        sts128(hb + kHtHBytes, make_uint4(lo[0], lo[1], lo[2], lo[3]));
        float* cb = bnd + col * 68;
#pragma unroll
        for (int k = 0; k < 8; ++k) rowsum = __fadd_ru(rowsum, fabsf(hv[k]));
        // sum_s |H_sd| over this thread's 8 s, then over the 4 chunk threads of row d.
        rowsum = __fadd_ru(rowsum, __shfl_xor_sync(0xffffffffu, rowsum, 1));
        rowsum = __fadd_ru(rowsum, __shfl_xor_sync(0xffffffffu, rowsum, 2));
        if (kc == 0) cb[32 + d] = rowsum;
        if (kc == (d >> 3)) cb[d] = hv[d & 7] >= 0.0f ? __fsqrt_ru(hv[d & 7]) : -1.0f;
        if (!strip_sync()) {
          ok = false;
          break;
        }
        // |H_sd| <= sqrt(H_ss) sqrt(H_dd) for every pair (true for a PSD H) lets
        // the tighter bound apply; checked on the rounded-up square roots.
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float ps = cb[8 * kc + k], pd = cb[d];
          cs = cs && ps >= 0.0f && pd >= 0.0f && fabsf(hv[k]) <= __fmul_ru(ps, pd);
        }
        cs = __all_sync(0xffffffffu, cs);
        if (lane == 0) reinterpret_cast<int*>(cb)[64 + quarter] = cs ? 1 : 0;
        fence_proxy_async_smem();
        if (!strip_sync()) {
          ok = false;
          break;
        }
      }
      const float* cb = bnd + col * 68;
      const int* csf = reinterpret_cast<const int*>(cb + 64);
      const bool use_cs = csf[0] && csf[1] && csf[2] && csf[3];

      // Anchor and candidate exponents (as quantize_block_fast).
      float amax, second;
      bool nonfinite;
      {
        const uint32_t lo1 = m1 & 0xffffu, hi1 = m1 >> 16;
        const uint32_t top1 = max(lo1, hi1);
        uint32_t top2 = 0;
        if constexpr (QM == kQTop2) top2 = max(min(lo1, hi1), max(m2 & 0xffffu, m2 >> 16));
        if constexpr (DT == MXW_BF16) {
          nonfinite = top1 >= 0x7f80u;
          amax = bits_f32(top1 << 16);
          second = bits_f32(top2 << 16);
        } else {
          nonfinite = top1 >= 0x7c00u;
          amax = __half2float(__ushort_as_half(static_cast<unsigned short>(top1)));
          second = __half2float(__ushort_as_half(static_cast<unsigned short>(top2)));
        }
      }
      unsigned long long unused_nt2[16];
      const float anchor = fmaxf(block_anchor<QM>(amax, second, unused_nt2, P), 1e-6f);
      const bool near_zero = amax < 1e-6f;
      bool fast = active && !near_zero && !nonfinite;
      const int f = fast ? floor_log2_div6(anchor) : 0;
      const int safe_e = fast ? ceil_log2_div6(fmaxf(amax, 1e-12f)) : 0;
      fast = fast && f <= 14 && safe_e <= f + 2;
      const int ncand = P.depth + 2 + (safe_e == f + 2 ? 1 : 0);
      const int amax_exp = static_cast<int>(f32_bits(amax) >> 23) - 127;  // floor(log2(amax)) for normal amax

      float best = __int_as_float(0x7f800000), best_tol = 0.0f;
      int best_c = 0;
      // Smallest E' - tol over the candidates other than the current best,
      // kept as the pair (E', tol) of every candidate seen: an ambiguity check
      // against the final best needs min over c != best of (E'_c - tol_c).
      float runner = __int_as_float(0x7f800000);  // min of E'_c - tol_c over c != best_c
      bool bad = false;
      // Rounds of up to kHtRound candidates, two in flight: round r + 1's D is
      // formed while round r's products are computed, and a buffer is refilled
      // (round r + 2) only after round r's epilogue has read it.
      const int64_t g0 = round;
      auto form = [&](int r) {
        const int buf = static_cast<int>((g0 + r) & 1);
#pragma unroll
        for (int cl = 0; cl < kHtRound; ++cl) {
          const int c = r * kHtRound + cl;
          if (c >= cmax) break;
          uint32_t dw[16];
          if (fast && c < ncand) {
            ht_candidate_d(words, c < P.depth + 2 ? f - P.depth + c : safe_e, dw);
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) dw[k] = 0u;
          }
          const uint32_t dst = my_d + buf * kHtDBuf + cl * kHtCols * kHtDBytes;
#pragma unroll
          for (int kc = 0; kc < 4; ++kc)
            sts128(dst + ht_core_offset(r_tile, kc), make_uint4(dw[4 * kc], dw[4 * kc + 1], dw[4 * kc + 2], dw[4 * kc + 3]));
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_ready[buf]);
      };
      auto epilogue = [&](int r) -> bool {
        const int64_t g = g0 + r;
        const int buf = static_cast<int>(g & 1);
        if (!__all_sync(0xffffffffu, mbar_wait(&mma_done[buf], static_cast<uint32_t>((g >> 1) & 1)))) return false;
        tc_fence_after();
#pragma unroll 1
        for (int cl = 0; cl < kHtRound; ++cl) {
          const int c = r * kHtRound + cl;
          if (c >= cmax) break;
          float w[32];
          tmem_ld_32x32b_x32(tl + buf * kHtTmemBuf + static_cast<uint32_t>((cl * kHtCols + col) * 32), w);
          if (!(fast && c < ncand)) continue;
          const uint32_t src = my_d + buf * kHtDBuf + cl * kHtCols * kHtDBytes;
          float e_sc, a_sc;
          if (use_cs) {
            ht_epilogue<true>(w, src, r_tile, cb, e_sc, a_sc);
          } else {
            ht_epilogue<false>(w, src, r_tile, cb, e_sc, a_sc);
          }
          // Back to the reference's units: E = E' * 2^(2e), exact for the
          // exponents here (-40 < e < 20).  D is exact in bf16 unless a clipped
          // element has |t| / 2^e >= 512 (then |x| - 6 needs more than 8 bits);
          // its rounding (2^-8 relative per element) enters the form twice.
          const int ec = c < P.depth + 2 ? f - P.depth + c : safe_e;
          const float s2 = exp2i(2 * ec);
          const float e_acc = __fmul_rn(e_sc, s2);
          const float tol = __fmul_ru(__fmul_ru(a_sc, s2), amax_exp - ec >= 9 ? kHtTolInexact : kHtTol);
          // A bound far down in the subnormal range no longer covers the
          // absolute rounding of the reference's intermediates: exact pass.
          if (isnan(e_acc) || !(tol < __int_as_float(0x7f800000)) || (a_sc > 0.0f && !(tol >= 0x1p-100f))) bad = true;
          if (e_acc < best) {
            runner = fminf(runner, __fsub_rd(best, best_tol));
            best = e_acc;
            best_tol = tol;
            best_c = c;
          } else {
            runner = fminf(runner, __fsub_rd(e_acc, tol));
          }
        }
        tc_fence_before();
        return true;
      };
      form(0);
      if (n_rounds > 1) form(1);
      for (int r = 0; r < n_rounds; ++r) {
        if (!epilogue(r)) {
          ok = false;
          break;
        }
        if (r + 2 < n_rounds) form(r + 2);
      }
      round = g0 + n_rounds;
      if (!ok) break;
      // Decided when every other candidate's lower end clears the best's upper end.
      const bool decided = fast && !bad && runner > __fadd_ru(best, best_tol);
      uint32_t sc;
      uint4 pk = make_uint4(0u, 0u, 0u, 0u);
      if (near_zero && active && !nonfinite) {
        sc = static_cast<uint32_t>(floor_log2_div6(anchor) - P.depth + 127);  // all-zero codes (core.py:194-195)
      } else if (decided) {
        const int raw = best_c < P.depth + 2 ? f - P.depth + best_c : safe_e;
        encode_pairs([&](int j) { return word_pair<DT>(words[j]); }, P, raw, pk);
        sc = static_cast<uint32_t>(raw + 127);
      } else {
        sc = kRareBlock;
      }
      if (active) {
        any_nonfinite |= nonfinite;
        any_rare |= sc == kRareBlock;
      }
      // Output.  A row's two block columns are adjacent 16-byte halves of one
      // 32-byte sector and two adjacent scale bytes: the column-1 warp of each
      // row quarter hands its half to the column-0 warp through shared memory,
      // and that warp writes both (half the store transactions, no partial
      // packed sectors).  Both hand-off waits are bounded.
      const int slot = quarter * 32 + lane;
      if (col == 1) {
        if (i > 0 && !__all_sync(0xffffffffu, mbar_wait(&pair_free[quarter], static_cast<uint32_t>((i - 1) & 1)))) {
          ok = false;
          break;
        }
        pair_pk[slot] = pk;
        pair_sc[slot] = sc;
        __syncwarp();
        if (lane == 0) mbar_arrive(&pair_ready[quarter]);
      } else {
        if (!__all_sync(0xffffffffu, mbar_wait(&pair_ready[quarter], static_cast<uint32_t>(i & 1)))) {
          ok = false;
          break;
        }
        const uint4 pk1 = pair_pk[slot];
        const uint32_t sc1 = pair_sc[slot];
        __syncwarp();
        if (lane == 0) mbar_arrive(&pair_free[quarter]);
        if (active) {
          const bool both = b + 1 < P.nb;
          uint8_t* dst = P.packed + row * (P.cols / 2) + b * 16;
          if (both && (reinterpret_cast<uintptr_t>(dst) & 31u) == 0) {
            asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(pk.x), "r"(pk.y),
                         "r"(pk.z), "r"(pk.w), "r"(pk1.x), "r"(pk1.y), "r"(pk1.z), "r"(pk1.w)
                         : "memory");
          } else {
            *reinterpret_cast<uint4*>(dst) = pk;
            if (both) *reinterpret_cast<uint4*>(dst + 16) = pk1;
          }
          uint8_t* sdst = P.scales + row * P.nb + b;
          if (both && (reinterpret_cast<uintptr_t>(sdst) & 1u) == 0) {
            *reinterpret_cast<uint16_t*>(sdst) = static_cast<uint16_t>((sc & 0xffu) | ((sc1 & 0xffu) << 8));
          } else {
            sdst[0] = static_cast<uint8_t>(sc);
            if (both) sdst[1] = static_cast<uint8_t>(sc1);
          }
        }
      }
    }
    if (P.flags && __any_sync(0xffffffffu, any_nonfinite) && lane == 0) atomicOr(P.flags, MXW_FLAG_NONFINITE);
    if (P.flags && __any_sync(0xffffffffu, any_rare) && lane == 0) atomicOr(P.flags, MXW_FLAG_RARE);
  }
  if (!ok && P.flags && lane == 0) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == kHtMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kHtTmemCols);
  }
}

// ------------------------- block-Hessian objective: exact pass for marked blocks
//
// The blocks the screening leaves undecided are re-quantized exactly, one
// warp per block: lane s holds element s, and lane d runs the reference's
// fp32 FMA chain w_d = sum_s dW_s H[s, d] over s = 0..31 (dW_s broadcast by
// shuffle, H[s, d] read as coalesced 128-byte rows and kept in registers for
// all candidates); the products fl(w_d dW_d) are then summed in the
// reference's 8-lane order (core.py:227-229).  A block whose elements are
// not all finite is left to the single-thread exact path.

__device__ __forceinline__ float warp_exact_hessian_error(float t, float dummy, int e, const float (&hcol)[32],
                                                          int lane) {
  (void)dummy;
  const float s = exp2i(e), inv = exp2i(-e);
  const float at = fabsf(t);
  const float xm = __fmul_rn(at, inv);  // |t| / 2^e (exact)
  uint32_t h2;
  asm("{\n\t.reg .b8 c;\n\tcvt.rn.satfinite.e2m1x2.f32 c, %1, %2;\n\tcvt.rn.f16x2.e2m1x2 %0, c;\n\t}"
      : "=r"(h2) : "f"(0.0f), "f"(xm));
  const float q = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xffffu)));
  // |dW| = q * 2^e - |t| (the product is exact unless it overflows, e >= 126), with t's sign.
  const float dwm = e < 126 ? __fmaf_rn(q, s, -at) : __fsub_rn(__fmul_rn(q, s), at);
  const float dw = __uint_as_float(__float_as_uint(dwm) ^ (__float_as_uint(t) & 0x80000000u));
  float w = 0.0f;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const float ds = __shfl_sync(0xffffffffu, dw, k);
    w = k == 0 ? __fmul_rn(ds, hcol[0]) : __fmaf_rn(ds, hcol[k], w);
  }
  const float prod = __fmul_rn(w, dw);
  // Lane partials ((p_l + p_{l+8}) + p_{l+16}) + p_{l+24}, then p_0 + ... + p_7 in order.
  float part = __fadd_rn(prod, __shfl_down_sync(0xffffffffu, prod, 8));
  part = __fadd_rn(part, __shfl_down_sync(0xffffffffu, prod, 16));
  part = __fadd_rn(part, __shfl_down_sync(0xffffffffu, prod, 24));
  float acc = __shfl_sync(0xffffffffu, part, 0);
#pragma unroll
  for (int l = 1; l < 8; ++l) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, part, l));
  (void)lane;
  return acc;
}

// One marked block (row, blk), the whole warp.  Mirrors quantize_one_block for
// the Hessian objective with a top-2 or amax anchor.
template <int DT, int QM>
__device__ __forceinline__ void warp_fixup_hessian_block(const QuantParams& P, int64_t idx, int lane) {
  const int64_t row = idx / P.nb, blk = idx % P.nb;
  float t;
  {
    const int64_t i = row * P.ld + blk * kBlock + lane;
    if constexpr (DT == MXW_BF16) {
      t = bits_f32(static_cast<uint32_t>(static_cast<const uint16_t*>(P.weight)[i]) << 16);
    } else if constexpr (DT == MXW_F16) {
      t = __half2float(static_cast<const __half*>(P.weight)[i]);
    } else {
      t = static_cast<const float*>(P.weight)[i];
    }
  }
  const uint32_t a = f32_bits(t) & 0x7fffffffu;
  // Non-finite elements: left marked for the single-thread exact pass, which
  // replays the reference's NaN handling.
  if (__any_sync(0xffffffffu, a >= 0x7f800000u)) return;
  // Top-2 magnitudes (ties: the second equals the first).
  const uint32_t m1 = __reduce_max_sync(0xffffffffu, a);
  const uint32_t n1 = __popc(__ballot_sync(0xffffffffu, a == m1));
  const uint32_t m2 = n1 >= 2 ? m1 : __reduce_max_sync(0xffffffffu, a == m1 ? 0u : a);
  const float amax = bits_f32(m1), second = bits_f32(m2);
  unsigned long long unused_nt2[16];
  float anchor = block_anchor<QM>(amax, second, unused_nt2, P);
  const bool near_zero = amax < 1e-6f;
  anchor = fmaxf(anchor, 1e-6f);
  const int floor_e = floor_log2_div6(anchor);
  const int lo_e = max(-127, min(127, floor_e - P.depth));
  uint32_t sc;
  uint32_t code = 0;
  if (near_zero) {
    sc = static_cast<uint32_t>(lo_e + 127);
  } else {
    const int hi_e = max(-127, min(127, floor_e + 1));
    const int safe_e = max(-127, min(127, ceil_log2_div6(fmaxf(amax, 1e-12f))));
    const int n_seq = hi_e - lo_e + 1;
    const bool safe_new = safe_e < lo_e || safe_e > hi_e;
    float hcol[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) hcol[k] = __ldg(P.hessian + blk * 1024 + k * 32 + lane);  // H[s = k][d = lane]
    float best = __int_as_float(0x7f800000);
    int raw = lo_e;
    for (int k = 0; k < n_seq + (safe_new ? 1 : 0); ++k) {
      const int e = k < n_seq ? lo_e + k : safe_e;
      const float err = warp_exact_hessian_error(t, 0.0f, e, hcol, lane);
      if (err < best) raw = e;
      best = (isnan(err) || isnan(best)) ? __int_as_float(0x7fffffff) : fminf(best, err);
    }
    // Final encode (core.py:242-249): x = t / 2^raw (+0 turns -0 into +0), E2M1 RNE.
    const float x = __fadd_rn(__fmul_rn(t, exp2i(-raw)), P.zero);
    const float xn = __shfl_down_sync(0xffffffffu, x, 1);
    code = e2m1x2(x, xn);  // meaningful in even lanes: elements (lane, lane + 1)
    sc = static_cast<uint32_t>(raw + 127);
  }
  // Bytes 0..15 from the even lanes; lane 4k assembles word k.
  const uint32_t b0 = __shfl_sync(0xffffffffu, code, (lane & ~3) * 2);
  const uint32_t b1 = __shfl_sync(0xffffffffu, code, (lane & ~3) * 2 + 2);
  const uint32_t b2 = __shfl_sync(0xffffffffu, code, (lane & ~3) * 2 + 4);
  const uint32_t b3 = __shfl_sync(0xffffffffu, code, (lane & ~3) * 2 + 6);
  uint8_t* dst = P.packed + row * (P.cols / 2) + blk * 16;
  if ((lane & 3) == 0 && lane < 16) {
    *reinterpret_cast<uint32_t*>(dst + lane) = (b0 & 0xffu) | ((b1 & 0xffu) << 8) | ((b2 & 0xffu) << 16) | ((b3 & 0xffu) << 24);
  }
  if (lane == 0) P.scales[idx] = static_cast<uint8_t>(sc);
}

// Finds the blocks quantize_hess_tc_kernel marked (scale byte kRareBlock) and
// re-quantizes each with a whole warp.  Each warp reads 512 scale bytes per
// step (16 per lane); returns at once when the main pass marked nothing.
template <int DT, int QM>
__global__ void __launch_bounds__(256, 4) quantize_fixup_hess_kernel(const QuantParams P) {
  if (P.flags && (*reinterpret_cast<volatile const uint32_t*>(P.flags) & MXW_FLAG_RARE) == 0) return;
  const int lane = threadIdx.x & 31;
  const int64_t total = P.rows * P.nb;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const bool vec = reinterpret_cast<uintptr_t>(P.scales) % 16 == 0;
  const int64_t span = vec ? 512 : 32;  // scale bytes per warp step
  for (int64_t base = warp * span; base < total; base += n_warps * span) {
    // Each lane's marked bytes as a bit mask over its 16 (or 1) positions.
    uint32_t mask = 0;
    if (vec) {
      const int64_t off = base + 16 * lane;
      if (off + 16 <= total) {
        const uint4 v = *reinterpret_cast<const uint4*>(P.scales + off);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t m = __vcmpeq4(w[q], 0xffffffffu);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if ((m >> (8 * k)) & 1u) mask |= 1u << (4 * q + k);
        }
      } else {
        for (int k = 0; k < 16 && off + k < total; ++k)
          if (P.scales[off + k] == kRareBlock) mask |= 1u << k;
      }
    } else if (base + lane < total && P.scales[base + lane] == kRareBlock) {
      mask = 1u;
    }
    uint32_t lanes = __ballot_sync(0xffffffffu, mask != 0);
    while (lanes) {
      const int src = __ffs(lanes) - 1;
      lanes &= lanes - 1;
      uint32_t m = __shfl_sync(0xffffffffu, mask, src);
      while (m) {
        const int k = __ffs(m) - 1;
        m &= m - 1;
        warp_fixup_hessian_block<DT, QM>(P, base + (vec ? 16 * src : src) + k, lane);
      }
    }
  }
}

// -------------------------------------------------- generic (unaligned) path

// One thread per block with plain loads: used when the input pointer or row
// stride cannot be described to TMA (16-byte rules).
template <int DT, int OBJ, int QM>
__global__ void __launch_bounds__(128) quantize_plain_kernel(const void* __restrict__ w, int64_t ld,
                                                             const QuantParams P) {
  const int64_t total = P.rows * P.nb;
  bool any_nonfinite = false;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / P.nb, b = idx % P.nb;
    BlockData<MXW_F32> B;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float x0, x1;
      if constexpr (DT == MXW_BF16) {
        const uint16_t* p = static_cast<const uint16_t*>(w) + r * ld + b * kBlock + 2 * j;
        x0 = bits_f32(static_cast<uint32_t>(p[0]) << 16);
        x1 = bits_f32(static_cast<uint32_t>(p[1]) << 16);
      } else if constexpr (DT == MXW_F16) {
        const __half* p = static_cast<const __half*>(w) + r * ld + b * kBlock + 2 * j;
        x0 = __half2float(p[0]);
        x1 = __half2float(p[1]);
      } else {
        const float* p = static_cast<const float*>(w) + r * ld + b * kBlock + 2 * j;
        x0 = p[0];
        x1 = p[1];
      }
      B.t2[j] = pack2(x0, x1);
    }
    // Order statistics on fp32 magnitude bits (exact for every input type).
    finish_stats_f32<MXW_F32, kQTop2>(B, B.t2);
    any_nonfinite |= B.nonfinite;
    unsigned long long g2[16];
    if constexpr (OBJ == kObjGamma) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float ga = P.gamma[b * kBlock + 2 * j], gb = P.gamma[b * kBlock + 2 * j + 1];
        g2[j] = pack2(__fmul_rn(ga, ga), __fmul_rn(gb, gb));
      }
    }
    uint4 pk;
    const uint32_t sc =
        quantize_one_block<MXW_F32, OBJ, QM, false>(B, P, g2, P.hessian ? P.hessian + b * 1024 : nullptr, pk);
    uint8_t* dst = P.packed + r * (P.cols / 2) + b * 16;
    const uint32_t words[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
    for (int k = 0; k < 16; ++k) dst[k] = static_cast<uint8_t>(words[k >> 2] >> (8 * (k & 3)));
    P.scales[r * P.nb + b] = static_cast<uint8_t>(sc);
  }
  if (P.flags && any_nonfinite) atomicOr(P.flags, MXW_FLAG_NONFINITE);
}

// --------------------------------------------------------------- host side

// Launch geometry per (kernel, device), computed once.
struct LaunchInfo {
  int per_sm = 0;
  bool smem_set = false;
};

static LaunchInfo& launch_info(const void* kern, int dev) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, LaunchInfo> cache;
  std::lock_guard<std::mutex> lock(mu);
  const uint64_t key = reinterpret_cast<uint64_t>(kern) ^ (static_cast<uint64_t>(dev) << 56);
  return cache[key];
}

template <int DT, int OBJ, int QM>
static int launch_tma(const void* w, int64_t ld, const QuantParams& P0, cudaStream_t stream) {
  const size_t smem = 1024 + kStages * Elem<DT>::kStageBytes + kOutBuffers * (kOutTileBytes + kScaleTileBytes) +
                      (OBJ == kObjHess ? kTileBlocks * 4096 : 0) + (OBJ == kObjGamma ? kTileBlocks * kGammaWords * 4 : 0) +
                      kTileBlocks * kBlock * 4 + (2 * kStages + 2 * kOutBuffers) * sizeof(uint64_t);
  CUtensorMap map;
  const CUtensorMapDataType dt = DT == MXW_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : DT == MXW_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if (make_tensor_map_2d(&map, dt, w, P0.cols, P0.rows, ld * Elem<DT>::kBytes, Elem<DT>::kBoxCols, kTileRows,
                         CU_TENSOR_MAP_SWIZZLE_128B) != MXW_OK)
    return MXW_ECUDA;
  CUtensorMap out_map;
  if (make_tensor_map_2d(&out_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, P0.packed, P0.cols / 2, P0.rows, P0.cols / 2,
                         kTileBlocks * 16, kTileRows, CU_TENSOR_MAP_SWIZZLE_128B) != MXW_OK)
    return MXW_ECUDA;
  auto kern = quantize_tma_kernel<DT, OBJ, QM>;
  int dev = 0;
  cudaGetDevice(&dev);
  LaunchInfo& li = launch_info(reinterpret_cast<const void*>(kern), dev);
  if (!li.smem_set) {
    const int rc = set_max_smem(reinterpret_cast<const void*>(kern), smem);
    if (rc != MXW_OK) return rc;
    int per_sm = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kQuantThreads, smem) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    li.per_sm = per_sm;
    li.smem_set = true;
  }
  QuantParams P = P0;
  P.n_tiles = ((P.nb + kTileBlocks - 1) / kTileBlocks) * P.n_row_tiles;
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(P.n_tiles, static_cast<int64_t>(num_sms()) * li.per_sm));
  kern<<<static_cast<unsigned>(ctas), kQuantThreads, smem, stream>>>(map, out_map, P);
  const int rc = check_launch();
  if constexpr (OBJ == kObjNone || OBJ == kObjGamma) {
    if (rc != MXW_OK) return rc;
    const int64_t chunks = (P.rows * P.nb + kFixupChunk - 1) / kFixupChunk;
    // One wave: at 255 registers a 256-thread CTA fills an SM, and the pass
    // is a grid-stride loop, so a second wave only adds launch cost to the
    // common case of a clear MXW_FLAG_RARE.
    const int64_t blocks = std::min<int64_t>((chunks + 255) / 256, static_cast<int64_t>(num_sms()));
    quantize_fixup_kernel<DT, OBJ, QM><<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), 256, 0, stream>>>(P, MXW_FLAG_RARE);
    return check_launch();
  }
  return rc;
}

// The block-Hessian objective on bf16 weights with a top-2 / amax anchor:
// tensor-core screening, then the rare-block pass for the blocks it leaves.
template <int DT, int QM>
static int launch_hess_tc(const void* w, int64_t ld, const QuantParams& P0, cudaStream_t stream) {
  CUtensorMap map;
  if (make_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, P0.cols, P0.rows, ld * 2, 64, kHtRows,
                         CU_TENSOR_MAP_SWIZZLE_128B) != MXW_OK)
    return MXW_ECUDA;
  auto kern = quantize_hess_tc_kernel<DT, QM>;
  int dev = 0;
  cudaGetDevice(&dev);
  LaunchInfo& li = launch_info(reinterpret_cast<const void*>(kern), dev);
  if (!li.smem_set) {
    const int rc = set_max_smem(reinterpret_cast<const void*>(kern), kHtSmem);
    if (rc != MXW_OK) return rc;
    li.per_sm = 2;
    li.smem_set = true;
  }
  QuantParams P = P0;
  P.n_row_tiles = (P.rows + kHtRows - 1) / kHtRows;
  const int64_t n_tiles = ((P.nb + kHtCols - 1) / kHtCols) * P.n_row_tiles;
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(n_tiles, static_cast<int64_t>(num_sms()) * li.per_sm));
  kern<<<static_cast<unsigned>(ctas), kHtThreads, kHtSmem, stream>>>(map, P);
  const int rc = check_launch();
  if (rc != MXW_OK) return rc;
  QuantParams F = P0;
  // One warp per 512 scale bytes, up to four 8-warp CTAs per SM: the marked
  // blocks spread over as many warps as the scan has steps.
  const int64_t steps = (F.rows * F.nb + 511) / 512;
  const int64_t blocks = std::min<int64_t>((steps + 7) / 8, static_cast<int64_t>(num_sms()) * 4);
  quantize_fixup_hess_kernel<DT, QM><<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), 256, 0, stream>>>(F);
  const int rc2 = check_launch();
  if (rc2 != MXW_OK) return rc2;
  // Blocks with non-finite elements (returns at once when the main pass saw none).
  const int64_t chunks = (F.rows * F.nb + kFixupChunk - 1) / kFixupChunk;
  const int64_t nf_blocks = std::min<int64_t>((chunks + 255) / 256, static_cast<int64_t>(num_sms()));
  quantize_fixup_kernel<DT, kObjHess, QM><<<static_cast<unsigned>(std::max<int64_t>(nf_blocks, 1)), 256, 0, stream>>>(
      F, MXW_FLAG_NONFINITE);
  return check_launch();
}

template <int DT, int OBJ, int QM>
static int launch_plain(const void* w, int64_t ld, const QuantParams& P, cudaStream_t stream) {
  const int64_t total = P.rows * P.nb;
  const int64_t blocks = std::min<int64_t>((total + 127) / 128, static_cast<int64_t>(num_sms()) * 16);
  quantize_plain_kernel<DT, OBJ, QM><<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), 128, 0, stream>>>(w, ld, P);
  return check_launch();
}

template <int DT, int OBJ, int QM>
static int launch_any(const void* w, int64_t ld, const QuantParams& P, cudaStream_t stream) {
  const bool tma_ok = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && ((ld * Elem<DT>::kBytes) % 16 == 0) &&
                      P.rows < (int64_t(1) << 31) && P.cols < (int64_t(1) << 31);
  if (tma_ok) return launch_tma<DT, OBJ, QM>(w, ld, P, stream);
  return launch_plain<DT, OBJ, QM>(w, ld, P, stream);
}

template <int DT, int OBJ>
static int dispatch_q(int qm, const void* w, int64_t ld, const QuantParams& P, cudaStream_t s) {
  if constexpr (OBJ == kObjHess && DT == MXW_BF16) {
    const bool tma_ok = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && ((ld * 2) % 16 == 0) &&
                        P.rows < (int64_t(1) << 31) && P.cols < (int64_t(1) << 31);
    if (tma_ok && qm == kQTop2) return launch_hess_tc<DT, kQTop2>(w, ld, P, s);
    if (tma_ok && qm == kQAmax) return launch_hess_tc<DT, kQAmax>(w, ld, P, s);
  }
  if (qm == kQAmax) return launch_any<DT, OBJ, kQAmax>(w, ld, P, s);
  if (qm == kQTop2) return launch_any<DT, OBJ, kQTop2>(w, ld, P, s);
  return launch_any<DT, OBJ, kQGeneral>(w, ld, P, s);
}

template <int DT>
static int dispatch_obj(int obj, int qm, const void* w, int64_t ld, const QuantParams& P, cudaStream_t s) {
  switch (obj) {
    case kObjNone:
      return dispatch_q<DT, kObjNone>(qm, w, ld, P, s);
    case kObjGamma:
      return dispatch_q<DT, kObjGamma>(qm, w, ld, P, s);
    case kObjHess:
      return dispatch_q<DT, kObjHess>(qm, w, ld, P, s);
    default:
      return launch_any<DT, kObjRtn, kQAmax>(w, ld, P, s);
  }
}

}  // namespace mxw
