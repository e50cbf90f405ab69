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
  kErrBarrierTimeout = 1,   // a bulk copy did not complete within the spin bound
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
// asynchronous bulk copies (TMA, non-tensor form) with an mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completion signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bounded wait on phase `parity`.  Every thread of the block must call it; returns
// false on every thread when any thread of the block gave up (error recorded).
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ bool block_wait(uint64_t* bar, uint32_t parity) {
  uint32_t n = 0;
  bool ok = false;
  while (n < kSpinLimit) {
    if (mbar_try_wait(bar, parity)) { ok = true; break; }
    ++n;
  }
  const int failed = __syncthreads_or(ok ? 0 : 1);
  if (failed) {
    raise_error(kErrBarrierTimeout);
    // give the copies in flight a second bounded chance to land before the
    // block's shared memory is released
    for (uint32_t m = 0; m < kSpinLimit && !mbar_try_wait(bar, parity); ++m) {}
    __syncthreads();
    return false;
  }
  return true;
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
// small utilities
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace gkv
