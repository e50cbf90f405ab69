// Device-side building blocks shared by the GraphKV sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/graphkv_b200.h"

namespace gkv {

// ---------------------------------------------------------------------------
// device error word (one per device; read and cleared by gkv_device_error)
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kErrNone = 0,
  kErrSelectCount = 2,      // selection produced list lengths different from the plan
  kErrBadIndex = 3,         // an index list entry outside [0, T)
};

// defined once: the library is a single translation unit (capi.cu)
__device__ int g_device_error = 0;

__device__ __forceinline__ void raise_error(int code) { atomicCAS(&g_device_error, 0, code); }

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kTag = GKV_F32;
  __device__ __forceinline__ static float to_f32(float x) { return x; }
  __device__ __forceinline__ static float from_f32(float x) { return x; }
};
template <> struct Elem<__half> {
  static constexpr int kTag = GKV_F16;
  __device__ __forceinline__ static float to_f32(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f32(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kTag = GKV_BF16;
  __device__ __forceinline__ static float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
};

// raw storage bits of one element
__device__ __forceinline__ uint32_t tbits(float x) { return __float_as_uint(x); }
__device__ __forceinline__ uint32_t tbits(__half x) { return __half_as_ushort(x); }
__device__ __forceinline__ uint32_t tbits(__nv_bfloat16 x) { return __bfloat16_as_ushort(x); }

// Store a float32 scale in the requested scale dtype (torch .to(), round to nearest even).
__device__ __forceinline__ void store_scale(void* base, int64_t i, int dtype, float s) {
  if (dtype == GKV_F16) reinterpret_cast<__half*>(base)[i] = __float2half_rn(s);
  else if (dtype == GKV_BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(s);
  else reinterpret_cast<float*>(base)[i] = s;
}
__device__ __forceinline__ float load_scale(const void* base, int64_t i, int dtype) {
  if (dtype == GKV_F16) return __half2float(reinterpret_cast<const __half*>(base)[i]);
  if (dtype == GKV_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}

// ---------------------------------------------------------------------------
// quantizer math (core.py:863-887), bit-exact with torch's fp32 CPU kernels
// ---------------------------------------------------------------------------
// torch compares and clamps fp32 tensors against the fp32 rounding of 1e-8.
constexpr float kEps = 1.0e-8f;
// 1.5 * 2^23: adding it to |a| < 2^22 rounds a to an integer (ties to even) in the
// low mantissa bits -- the same rounding torch.round performs.
constexpr float kMagic = 12582912.0f;

struct GroupCoder {
  float scale;   // fp32 scale used for coding (before the cast to the scale dtype)
  float inv;     // correctly rounded 1 / scale
  float lo, hi;  // clamp range of the quotient (symmetric) or of quotient + zp (affine)
  float zp;      // zero point as float (0 for symmetric)
  int zpi;
  float magic;   // kMagic + encoding offset
};

// Symmetric: scale = max(absmax, eps) / qmax; codes in [qmin, qmax]; stored code - qmin
// when packed, the raw int8 otherwise.
__device__ __forceinline__ GroupCoder make_symmetric(float absmax, int bits, bool packed) {
  GroupCoder c;
  const int qmax = (1 << (bits - 1)) - 1;
  const int qmin = -(1 << (bits - 1));
  c.scale = __fdiv_rn(fmaxf(absmax, kEps), (float)qmax);
  c.inv = __frcp_rn(c.scale);
  c.lo = (float)qmin;
  c.hi = (float)qmax;
  c.zp = 0.f;
  c.zpi = 0;
  c.magic = kMagic + (packed ? (float)(-qmin) : 0.f);
  return c;
}

// Affine: scale from the range (or the absmax when the range is degenerate);
// zero point round(-min / scale) clamped to [0, qmax] (core.py:863-880).
__device__ __forceinline__ GroupCoder make_affine(float mn, float mx, int bits) {
  GroupCoder c;
  const int qmax = (1 << bits) - 1;
  const float range = __fsub_rn(mx, mn);
  const bool degenerate = range < kEps;
  const float absmax = fmaxf(fabsf(mn), fabsf(mx));
  c.scale = degenerate ? __fdiv_rn(fmaxf(absmax, kEps), (float)qmax) : __fdiv_rn(fmaxf(range, kEps), (float)qmax);
  if (degenerate) {
    c.zpi = mn < 0.f ? qmax : 0;
  } else {
    float z = rintf(__fdiv_rn(-mn, c.scale));
    z = fminf(fmaxf(z, 0.f), (float)qmax);
    c.zpi = (int)z;
  }
  c.zp = (float)c.zpi;
  c.inv = __frcp_rn(c.scale);
  c.lo = 0.f;
  c.hi = (float)qmax;
  c.magic = kMagic;
  return c;
}

// Exact code of one element: round_half_even(fl(fl(x / scale) [+ zp])) clamped.
// Fast path multiplies by the reciprocal: |x * inv - x / scale| < 2^-22 |x / scale|,
// so the rounded integer can only differ when x * inv lies within that distance of a
// half-integer; those elements take the IEEE division.  Returns the encoded byte value.
__device__ __forceinline__ uint32_t code_of(float x, const GroupCoder& c) {
  float a = __fmul_rn(x, c.inv);
  const float r = __fsub_rn(__fadd_rn(a, kMagic), kMagic);  // rint(a) for |a| < 2^22
  const float d = fabsf(__fsub_rn(a, r));
  const float tol = __fmaf_rn(fabsf(a), 9.5367431640625e-07f /*2^-20*/, 3.814697265625e-06f /*2^-18*/);
  if (d > 0.5f - tol || !(fabsf(a) < 4194304.0f)) {
    a = __fdiv_rn(x, c.scale);  // exact quotient, the reference's operation
  }
  a = __fadd_rn(a, c.zp);
  a = fminf(fmaxf(a, c.lo), c.hi);
  const float t = __fadd_rn(a, c.magic);
  return __float_as_uint(t) - __float_as_uint(kMagic);
}

// ---------------------------------------------------------------------------
// Packed fp32 pairs (sm_100 f32x2 arithmetic: two IEEE round-to-nearest
// operations per instruction, bitwise the same as two scalar ones)
// ---------------------------------------------------------------------------
// A register pair from two 32-bit values, and its halves (register moves only).
__device__ __forceinline__ uint64_t pk2u(uint32_t a, uint32_t b) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t lo32(uint64_t v) {
  uint32_t a;
  asm("{\n\t.reg .b32 h;\n\tmov.b64 {%0, h}, %1;\n\t}" : "=r"(a) : "l"(v));
  return a;
}
__device__ __forceinline__ uint32_t hi32(uint64_t v) {
  uint32_t b;
  asm("{\n\t.reg .b32 l;\n\tmov.b64 {l, %0}, %1;\n\t}" : "=r"(b) : "l"(v));
  return b;
}
__device__ __forceinline__ uint64_t pk2(float a, float b) { return pk2u(__float_as_uint(a), __float_as_uint(b)); }
__device__ __forceinline__ float lo2(uint64_t v) { return __uint_as_float(lo32(v)); }
__device__ __forceinline__ float hi2(uint64_t v) { return __uint_as_float(hi32(v)); }
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// ---------------------------------------------------------------------------
// Packed encoding of a run of N (even) elements of one group.
//
// Quotient: the reference rounds fl(x / scale) to an integer (core.py:879, 886).
// With y = fl(1 / scale) (correctly rounded reciprocal), q0 = fl(x * y),
// r = fl(x - q0 * scale) and q = fl(q0 + r * y) (two fused multiply-adds; the
// quotient correction of P. Markstein, "Computation of elementary functions on the
// IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990) equals the IEEE
// quotient except for |x / scale| < 2^-79, where both round to the same code.  This
// was checked against the IEEE division on 2.7e10 (x, scale) pairs: every bf16 and
// fp16 x against every scale a bf16 / fp16 group maximum yields for
// qmax in {1, 3, 7, 15, 127, 255}, and random fp32 pairs, with identical codes for
// the symmetric rounding and for every affine zero point.
//
// Per pair of elements: q as above, [+ zp, clamped to [0, qmax] for affine];
// t = fl(q + magic) holds the code in its low mantissa bits (bits(t) =
// bits(kMagic) + code, ties to even as torch.round).  Codes are packed
// little-end-first by Horner steps acc = acc * 2^SB + bits(t) (mod 2^32); the
// constant contribution of bits(kMagic) is subtracted once per word.
// ---------------------------------------------------------------------------
struct FastCoder {
  float scale;  // fp32 coding scale
  float inv;    // fl(1 / scale)
  float zp;     // affine zero point (0 for symmetric)
  float hi;     // affine clamp: qmax
  float magic;  // kMagic + offset: packed symmetric -qmin, unpacked symmetric 128, affine 0
  uint32_t flip;  // per-byte XOR applied to unpacked symmetric codes (0x80808080) or 0
};

// sum over the first `cnt` element slots of a word of bits(kMagic) << (SB * i), mod 2^32
template <int SB>
__host__ __device__ constexpr uint32_t magic_sum(int cnt) {
  uint32_t s = 0;
  for (int i = 0; i < cnt; ++i) s += 0x4B400000u << (SB * i);
  return s;
}

// per-byte flip restricted to the bytes of `cnt` slots
template <int SB>
__host__ __device__ constexpr uint32_t slot_mask(int cnt) {
  return cnt * SB >= 32 ? 0xFFFFFFFFu : ((1u << (cnt * SB)) - 1u);
}

// ---------------------------------------------------------------------------
// Correctly rounded quotient x / c from rc = RN(1 / c): one product and one
// fused-multiply-add correction (Markstein).  For the divisors used here -- the
// code ranges qmax in {3, 7, 15, 127, 255} and fp32(sqrt(D)) for D in
// {32, 128, 512} -- this equals the IEEE quotient for every fp32 x whose
// quotient is at least 2^-100 in magnitude (checked exhaustively over all 2^32
// bit patterns against __fdiv_rn); qmax = 1 and powers of two are exact trivially.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float quot(float x, float c, float rc) {
  const float q0 = __fmul_rn(x, rc);
  return __fmaf_rn(__fmaf_rn(-q0, c, x), rc, q0);
}
__device__ __forceinline__ uint64_t quot2(uint64_t x2, uint64_t nc2, uint64_t rc2) {
  const uint64_t q0 = mul2(x2, rc2);
  return fma2(fma2(q0, nc2, x2), rc2, q0);
}

// Group coders built from a group's statistics (core.py:863-887); the scale
// division by qmax uses quot() (exact for every scale >= 1e-8).
__device__ __forceinline__ FastCoder sym_coder(float absmax, float qmax, float rqmax, int bits, bool packed) {
  FastCoder c;
  c.scale = quot(fmaxf(absmax, kEps), qmax, rqmax);
  c.inv = __frcp_rn(c.scale);
  c.zp = 0.f;
  c.hi = qmax;
  if (packed) {
    c.magic = kMagic + (float)(1 << (bits - 1));
    c.flip = 0u;
  } else {
    c.magic = kMagic + 128.f;
    c.flip = 0x80808080u;
  }
  return c;
}

__device__ __forceinline__ FastCoder aff_coder(float mn, float mx, float qmax, float rqmax) {
  FastCoder c;
  const float range = __fsub_rn(mx, mn);
  const bool degenerate = range < kEps;
  const float absmax = fmaxf(fabsf(mn), fabsf(mx));
  c.scale = quot(fmaxf(degenerate ? absmax : range, kEps), qmax, rqmax);
  c.inv = __frcp_rn(c.scale);
  float z;
  if (degenerate) {
    z = mn < 0.f ? qmax : 0.f;
  } else {
    // round(-min / scale): the quotient from the reciprocal, corrected once,
    // rounds like the IEEE quotient (the same argument as for the codes)
    z = fminf(fmaxf(rintf(quot(-mn, c.scale, c.inv)), 0.f), qmax);
  }
  c.zp = z;
  c.hi = qmax;
  c.magic = kMagic;
  c.flip = 0u;
  return c;
}

// ---------------------------------------------------------------------------
// Packed statistics of 32-bit words holding two 16-bit elements.
// max.xorsign.abs returns max(|a|, |b|) with the XOR of the signs: the
// magnitude accumulates the absolute maximum of both halves independently.
// ---------------------------------------------------------------------------
template <typename T> struct Word16;
template <> struct Word16<__nv_bfloat16> {
  __device__ __forceinline__ static uint32_t amax(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t vmax(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t vmin(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  // packed minimum of magnitudes (the result's sign is the XOR of the signs)
  __device__ __forceinline__ static uint32_t amin(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static constexpr uint32_t kNegInf = 0xFF80FF80u, kPosInf = 0x7F807F80u, kMaxFinite = 0x7F7F7F7Fu;
  __device__ __forceinline__ static float lo(uint32_t w) { return __uint_as_float(w << 16); }
  __device__ __forceinline__ static float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
  __device__ __forceinline__ static uint64_t pair(uint32_t w) { return pk2(lo(w), hi(w)); }
  __device__ __forceinline__ static uint32_t round2(float a, float b) {  // (a low, b high), RNE
    const __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&r);
  }
};
template <> struct Word16<__half> {
  __device__ __forceinline__ static uint32_t amax(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t vmax(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t vmin(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t amin(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static constexpr uint32_t kNegInf = 0xFC00FC00u, kPosInf = 0x7C007C00u, kMaxFinite = 0x7BFF7BFFu;
  __device__ __forceinline__ static float lo(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
  }
  __device__ __forceinline__ static float hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
  __device__ __forceinline__ static uint64_t pair(uint32_t w) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    return pk2(f.x, f.y);
  }
  __device__ __forceinline__ static uint32_t round2(float a, float b) {
    const __half2 r = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&r);
  }
};

// ---------------------------------------------------------------------------
// Fast Walsh-Hadamard butterflies of a row spread over a warp, lane holding EPL
// consecutive elements.  Stages run in the reference order h = 1, 2, 4, ...
// (core.py:950-955); every output is one fp32 add or subtract of the previous
// stage, as there.  Cross-lane stages compute o + sign * v with one fused
// multiply-add (sign +1: v + o on the left lane, -1: o - v on the right lane).
// ---------------------------------------------------------------------------
template <int EPL>
__device__ __forceinline__ void fwht_warp(float (&v)[EPL]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = 1; h < EPL; h <<= 1) {
    if constexpr (EPL >= 4) {
      // two butterflies per packed add / subtract
#pragma unroll
      for (int i = 0; i < EPL; i += 2 * h) {
#pragma unroll
        for (int j = 0; j < h; j += 2) {
          const int a = i + j;
          if (h == 1) {
            // pairs (a, a+1) and (a+2, a+3)
            if ((a & 3) != 0) continue;
            const uint64_t l = pk2(v[a], v[a + 2]), r = pk2(v[a + 1], v[a + 3]);
            const uint64_t s = add2(l, r), df = sub2(l, r);
            v[a] = lo2(s); v[a + 2] = hi2(s); v[a + 1] = lo2(df); v[a + 3] = hi2(df);
          } else {
            const uint64_t l = pk2(v[a], v[a + 1]), r = pk2(v[a + h], v[a + h + 1]);
            const uint64_t s = add2(l, r), df = sub2(l, r);
            v[a] = lo2(s); v[a + 1] = hi2(s); v[a + h] = lo2(df); v[a + h + 1] = hi2(df);
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        if ((i & h) == 0) {
          const float a = v[i], b = v[i + h];
          v[i] = __fadd_rn(a, b);
          v[i + h] = __fsub_rn(a, b);
        }
      }
    }
  }
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const float sg = (lane & m) ? -1.f : 1.f;
    const uint64_t sg2 = pk2(sg, sg);
#pragma unroll
    for (int i = 0; i < EPL; i += 2) {
      const float o0 = __shfl_xor_sync(0xFFFFFFFFu, v[i], m);
      const float o1 = __shfl_xor_sync(0xFFFFFFFFu, v[i + 1], m);
      const uint64_t r = fma2(sg2, pk2(v[i], v[i + 1]), pk2(o0, o1));
      v[i] = lo2(r);
      v[i + 1] = hi2(r);
    }
  }
}

constexpr unsigned kFull = 0xFFFFFFFFu;

// In-register Hadamard transform of one row split into RPR runs of RUN elements
// held by the lanes 8 apart (run u in lane bits 3-4).  Butterflies h = 1 .. RUN/2
// inside the thread, h >= RUN across lanes, in the reference order; then y / div.
// CHECK: the fused quotient when `fused` (proven exact for quotients >= 2^-100)
// and no |y| of this thread is below 2^-90 (zeros included: the fused form turns
// -0 into +0), else IEEE division.  Without CHECK the caller guarantees that
// every nonzero y is far above 2^-90 and that no y is -0, and `fused` selects.
template <int RUN, int RPR, bool CHECK = true>
__device__ __forceinline__ void rotate_run(uint64_t (&v)[RUN / 2], int u, float div, float rdiv, bool fused) {
  // h = 1: inside each pair
#pragma unroll
  for (int k = 0; k < RUN / 2; ++k) {
    const float a = lo2(v[k]), b = hi2(v[k]);
    v[k] = pk2(__fadd_rn(a, b), __fsub_rn(a, b));
  }
  // h = 2 .. RUN/2: pairs k and k + h/2
#pragma unroll
  for (int h = 2; h < RUN; h <<= 1) {
#pragma unroll
    for (int k = 0; k < RUN / 2; ++k) {
      if ((2 * k) & h) continue;
      const uint64_t a = v[k], b = v[k + h / 2];
      v[k] = add2(a, b);
      v[k + h / 2] = sub2(a, b);
    }
  }
  // h = RUN .. (RPR * RUN) / 2: across lanes
  // (left lane: v + o; right lane: o - v, as fma(-1, v, o): one rounding, as the subtraction)
#pragma unroll
  for (int m = 1; m < RPR; m <<= 1) {
    const float sg = (u & m) ? -1.f : 1.f;
    const uint64_t sg2 = pk2(sg, sg);
#pragma unroll
    for (int k = 0; k < RUN / 2; ++k) {
      const float o0 = __shfl_xor_sync(kFull, lo2(v[k]), 8 * m);
      const float o1 = __shfl_xor_sync(kFull, hi2(v[k]), 8 * m);
      v[k] = fma2(sg2, v[k], pk2(o0, o1));
    }
  }
  if constexpr (CHECK) {
    float least = __int_as_float(0x7f800000);
#pragma unroll
    for (int k = 0; k < RUN / 2; ++k) least = fminf(least, fminf(fabsf(lo2(v[k])), fabsf(hi2(v[k]))));
    fused = fused && !(least < 8.077935669463161e-28f /* 2^-90 */);
  }
  if (fused) {
    const uint64_t nd2 = pk2(-div, -div), rd2 = pk2(rdiv, rdiv);
#pragma unroll
    for (int k = 0; k < RUN / 2; ++k) v[k] = quot2(v[k], nd2, rd2);
  } else {
#pragma unroll
    for (int k = 0; k < RUN / 2; ++k) v[k] = pk2(__fdiv_rn(lo2(v[k]), div), __fdiv_rn(hi2(v[k]), div));
  }
}

// ---------------------------------------------------------------------------
// Hadamard helpers (core.py:945-956)
// ---------------------------------------------------------------------------
// y / divisor rounded to T.  For bf16 a product with the reciprocal is accurate to a
// few fp32 ulps; only values within a few ulps of a bf16 rounding midpoint need the
// exact division.  Other dtypes always divide.
template <typename T>
__device__ __forceinline__ T hadamard_scale(float y, float divisor, float inv_divisor) {
  if constexpr (Elem<T>::kTag == GKV_BF16) {
    const float z = __fmul_rn(y, inv_divisor);
    const uint32_t low = __float_as_uint(z) & 0xFFFFu;
    const int dist = (int)low - 0x8000;
    const float q = (dist > 8 || dist < -8) ? z : __fdiv_rn(y, divisor);
    return Elem<T>::from_f32(q);
  } else {
    return Elem<T>::from_f32(__fdiv_rn(y, divisor));
  }
}

// ---------------------------------------------------------------------------
// asynchronous 16-byte copies into shared memory
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous global -> shared copy; src_bytes == 0 writes zeros
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)), "l"(src), "r"(src_bytes)
               : "memory");
}

// ---------------------------------------------------------------------------
// vector stores
// ---------------------------------------------------------------------------
// store NB bytes (power of two, 1..32) from words w[] at an NB-aligned address
template <int NB>
__device__ __forceinline__ void store_bytes(uint8_t* dst, const uint32_t* w) {
  if constexpr (NB == 1) {
    *dst = (uint8_t)w[0];
  } else if constexpr (NB == 2) {
    *reinterpret_cast<uint16_t*>(dst) = (uint16_t)w[0];
  } else if constexpr (NB == 4) {
    *reinterpret_cast<uint32_t*>(dst) = w[0];
  } else if constexpr (NB == 8) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  } else if constexpr (NB == 16) {
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    static_assert(NB == 32, "store size");
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(dst + 16) = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

// ---------------------------------------------------------------------------
// Code extraction: 2^23 + code as an fp32 bit pattern, one byte permute per code.
// `nib[k]` holds code k of a word in the low byte of byte k' of one of the masked
// words below; PRMT places that byte under the exponent byte 0x4B.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t with_magic(uint32_t src, int byte) {
  return __byte_perm(src, 0x4B000000u, 0x7540u | (uint32_t)byte);
}

// 32 / SB codes of one 32-bit word, in element order, as fp32 bit patterns 2^23 + code
template <int SB>
__device__ __forceinline__ void word_codes(uint32_t w, uint32_t (&out)[32 / SB]) {
  if constexpr (SB == 8) {
#pragma unroll
    for (int k = 0; k < 4; ++k) out[k] = with_magic(w, k);
  } else if constexpr (SB == 4) {
    const uint32_t ev = w & 0x0F0F0F0Fu, od = (w >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      out[2 * k] = with_magic(ev, k);
      out[2 * k + 1] = with_magic(od, k);
    }
  } else {
    uint32_t m[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) m[j] = (w >> (2 * j)) & 0x03030303u;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) out[4 * k + j] = with_magic(m[j], k);
  }
}

// ---------------------------------------------------------------------------
// small utilities
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace gkv
