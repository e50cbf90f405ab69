// Unpack + dequantize + scatter kernels (core.py:153-173, 265-307, 993-1007).
//
// Every output row [s, t, :] is written exactly once: retained rows are copied
// from the retained store, standard and cold rows are decoded from their tiers.
// Decoded values are (q - zp) * scale in fp32 (one rounding, no FMA), then the
// optional inverse Hadamard (the same butterflies, fp32), then the cast to the
// cache dtype.
//
// Fast path: one block per tile of TT tier rows of one slice.  Token-axis
// tensors decode a [TT, D] fp32 tile in shared memory (thread per channel and
// run of 16 rows), channel-axis tensors decode straight from the packed rows
// (warp per row); both leave through warp-per-row stores of whole output rows.
#pragma once

#include "gkv_params.cuh"

namespace gkv {

// Decode offset: value = float((enc ^ xor_mask) + off) reproduces the reference's
// unpack (core.py:993-1007) -- enc + qmin for packed symmetric codes, the int8 for
// unpacked symmetric codes, and enc - zp for affine codes.
struct Decoder {
  uint32_t xor_mask;
  float base;   // 2^23 - off: float(2^23 + x) - base == x + off exactly
  float scale;
};

__device__ __forceinline__ Decoder make_decoder(const TensorDesc& d, float scale, int zp) {
  Decoder r;
  r.scale = scale;
  if (d.quantizer == GKV_AFFINE) {
    r.xor_mask = 0;
    r.base = 8388608.0f + (float)zp;
  } else if (d.packed) {
    r.xor_mask = 0;
    r.base = 8388608.0f + (float)(1 << (d.bits - 1));  // enc + qmin
  } else {
    r.xor_mask = 0x80u;                                 // int8 two's complement
    r.base = 8388608.0f + 128.0f;
  }
  return r;
}

__device__ __forceinline__ float decode(uint32_t enc, const Decoder& dc) {
  const float q = __fsub_rn(__uint_as_float(0x4B000000u | (enc ^ dc.xor_mask)), dc.base);
  return __fmul_rn(q, dc.scale);
}

__device__ __forceinline__ int load_zp(const TensorDesc& d, int64_t gi) {
  return d.quantizer == GKV_AFFINE ? (int)d.zps[gi] : 0;
}

// Output of one decoded row: optional inverse rotation across the warp, cast, store.
template <typename T, int D>
__device__ __forceinline__ void emit_row(float (&v)[D / 32], bool rotate, float div, float inv, T* dst) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  if (rotate) {
#pragma unroll
    for (int h = 1; h < EPL; h <<= 1) {
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        if ((i & h) == 0) {
          const float a = v[i], b = v[i + h];
          v[i] = __fadd_rn(a, b);
          v[i + h] = __fsub_rn(a, b);
        }
      }
    }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const bool right = (lane & m) != 0;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const float o = __shfl_xor_sync(0xFFFFFFFFu, v[i], m);
        v[i] = right ? __fsub_rn(o, v[i]) : __fadd_rn(v[i], o);
      }
    }
  }
  constexpr int NB = EPL * (int)sizeof(T);
  constexpr int NW = NB / 4;
  uint32_t w[NW];
#pragma unroll
  for (int q = 0; q < NW; ++q) w[q] = 0;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const T o = rotate ? hadamard_scale<T>(v[i], div, inv) : Elem<T>::from_f32(v[i]);
    w[(i * (int)sizeof(T)) / 4] |= tbits(o) << (((i * (int)sizeof(T)) % 4) * 8);
  }
  store_bytes<NB>(reinterpret_cast<uint8_t*>(dst + lane * EPL), w);
}

// load NBITS (power of two <= 64) bits starting at bit offset `bit` (aligned to NBITS)
template <int NBITS>
__device__ __forceinline__ uint64_t load_bits(const uint8_t* codes, int64_t bit) {
  if constexpr (NBITS <= 8) {
    return (uint64_t)((codes[bit >> 3] >> (bit & 7)) & ((1u << NBITS) - 1u));
  } else if constexpr (NBITS == 16) {
    return reinterpret_cast<const uint16_t*>(codes)[bit >> 4];
  } else if constexpr (NBITS == 32) {
    return reinterpret_cast<const uint32_t*>(codes)[bit >> 5];
  } else {
    return reinterpret_cast<const uint64_t*>(codes)[bit >> 6];
  }
}

// channel-axis tensor: warp per tier row
template <typename T, int D, int SB>
__device__ void dequant_channel_tile(const DequantParams& p, const TensorDesc& d, T* out, const int* idx, int s,
                                     int j0, int rows) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = warp; r < rows; r += kThreads / 32) {
    const int64_t row = (int64_t)s * d.n + j0 + r;
    const uint64_t bits = load_bits<EPL * SB>(d.codes, (row * d.n_pad + lane * EPL) * SB);
    const int64_t gi = row * d.groups_row + ((lane * EPL) >> d.log2gs);
    const Decoder dc = make_decoder(d, load_scale(d.scales, gi, d.scale_dtype), load_zp(d, gi));
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = decode((uint32_t)(bits >> (i * SB)) & ((1u << SB) - 1u), dc);
    const int tok = idx[j0 + r];
    if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); continue; }
    emit_row<T, D>(v, d.rotation != 0, p.had_div, p.had_inv, out + (int64_t)tok * D);
  }
}

// token-axis tensor: decode the tile into shared memory, then warp-per-row stores
template <typename T, int D, int TT, int SB>
__device__ void dequant_token_tile(const DequantParams& p, const TensorDesc& d, T* out, const int* idx, int s, int j0,
                                   int rows, float* tile) {
  constexpr int PARTS = kThreads / D;
  constexpr int PR = TT / PARTS;
  constexpr int TP = D + 4;  // fp32 pitch
  const int c = threadIdx.x % D, part = threadIdx.x / D;
  const int64_t crow = (int64_t)s * D + c;
#pragma unroll
  for (int q = 0; q < PR / 16; ++q) {
    const int r0 = part * PR + q * 16;
    const int tok = j0 + r0;
    if (tok < d.n_pad) {
      const int64_t gi = crow * d.groups_row + (tok >> d.log2gs);
      const Decoder dc = make_decoder(d, load_scale(d.scales, gi, d.scale_dtype), load_zp(d, gi));
      const int64_t bit = (crow * d.n_pad + tok) * SB;
      uint32_t w[SB / 2];  // 16 codes
      if constexpr (SB == 2) {
        w[0] = reinterpret_cast<const uint32_t*>(d.codes)[bit >> 5];
      } else if constexpr (SB == 4) {
        const uint2 t = reinterpret_cast<const uint2*>(d.codes)[bit >> 6];
        w[0] = t.x; w[1] = t.y;
      } else {
        const uint4 t = reinterpret_cast<const uint4*>(d.codes)[bit >> 7];
        w[0] = t.x; w[1] = t.y; w[2] = t.z; w[3] = t.w;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t enc = (w[(i * SB) / 32] >> ((i * SB) % 32)) & ((1u << SB) - 1u);
        tile[(r0 + i) * TP + c] = decode(enc, dc);
      }
    }
  }
  __syncthreads();
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = warp; r < rows; r += kThreads / 32) {
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = tile[r * TP + lane * EPL + i];
    const int tok = idx[j0 + r];
    if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); continue; }
    emit_row<T, D>(v, d.rotation != 0, p.had_div, p.had_inv, out + (int64_t)tok * D);
  }
  __syncthreads();
}

template <typename T, int D, int TT>
__device__ __forceinline__ void dequant_tensor(const DequantParams& p, const TensorDesc& d, T* out, const int* idx,
                                               int s, int j0, int rows, float* tile) {
  if (d.axis == GKV_AXIS_TOKEN) {
    if (d.sbits == 4) dequant_token_tile<T, D, TT, 4>(p, d, out, idx, s, j0, rows, tile);
    else if (d.sbits == 2) dequant_token_tile<T, D, TT, 2>(p, d, out, idx, s, j0, rows, tile);
    else dequant_token_tile<T, D, TT, 8>(p, d, out, idx, s, j0, rows, tile);
  } else {
    if (d.sbits == 4) dequant_channel_tile<T, D, 4>(p, d, out, idx, s, j0, rows);
    else if (d.sbits == 2) dequant_channel_tile<T, D, 2>(p, d, out, idx, s, j0, rows);
    else dequant_channel_tile<T, D, 8>(p, d, out, idx, s, j0, rows);
  }
}

template <typename T, int D, int TT>
constexpr size_t dequant_tile_smem() {
  return (size_t)TT * (D + 4) * sizeof(float);
}

template <typename T, int D, int TT>
__global__ void __launch_bounds__(kThreads) dequantize_tile_kernel(const __grid_constant__ DequantParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  float* tile = reinterpret_cast<float*>(smem);
  const int s = blockIdx.x / p.tiles_slice;
  int k = blockIdx.x - s * p.tiles_slice;
  T* ok = reinterpret_cast<T*>(p.out_k) + (int64_t)s * p.T * D;
  T* ov = reinterpret_cast<T*>(p.out_v) + (int64_t)s * p.T * D;
  if (k < p.tiles[0]) {
    constexpr int VEC = 16 / (int)sizeof(T), CPR = D / VEC;
    const int R = p.n_tier[0];
    const int j0 = k * kRetTile, rows = min(kRetTile, R - j0);
    const T* rk = reinterpret_cast<const T*>(p.ret_k) + ((int64_t)s * R + j0) * D;
    const T* rv = reinterpret_cast<const T*>(p.ret_v) + ((int64_t)s * R + j0) * D;
    for (int e = threadIdx.x; e < rows * CPR; e += kThreads) {
      const int r = e / CPR, c = e - r * CPR;
      const int tok = p.idx[0][j0 + r];
      if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); continue; }
      *reinterpret_cast<uint4*>(ok + (int64_t)tok * D + c * VEC) = *reinterpret_cast<const uint4*>(rk + r * D + c * VEC);
      *reinterpret_cast<uint4*>(ov + (int64_t)tok * D + c * VEC) = *reinterpret_cast<const uint4*>(rv + r * D + c * VEC);
    }
    return;
  }
  k -= p.tiles[0];
  int tier = 1;
  if (k >= p.tiles[1]) { k -= p.tiles[1]; tier = 2; }
  const TensorDesc& dk = p.t[tier == 1 ? GKV_STD_K : GKV_COLD_K];
  const TensorDesc& dv = p.t[tier == 1 ? GKV_STD_V : GKV_COLD_V];
  const int* idx = p.idx[tier];
  const int j0 = k * TT;
  const int rows = min(TT, p.n_tier[tier] - j0);
  dequant_tensor<T, D, TT>(p, dk, ok, idx, s, j0, rows, tile);
  dequant_tensor<T, D, TT>(p, dv, ov, idx, s, j0, rows, tile);
}

// ---------------------------------------------------------------------------
// general path: warp per tier row (both K and V), element-wise decode
// ---------------------------------------------------------------------------
__device__ __forceinline__ float decode_element(const TensorDesc& d, int64_t e, int64_t gi) {
  const int64_t bit = e * d.sbits;
  const uint32_t enc = (d.codes[bit >> 3] >> (bit & 7)) & ((1u << d.sbits) - 1u);
  return decode(enc, make_decoder(d, load_scale(d.scales, gi, d.scale_dtype), load_zp(d, gi)));
}

template <typename T>
__global__ void __launch_bounds__(256) general_dequant_rows_kernel(const __grid_constant__ DequantParams p, int tier) {
  extern __shared__ float gbuf[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = p.n_tier[tier];
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= (int64_t)p.S * n) return;
  const int s = (int)(row / n), j = (int)(row % n);
  const int D = p.D;
  const int tok = p.idx[tier][j];
  if ((unsigned)tok >= (unsigned)p.T) { if (lane == 0) raise_error(kErrBadIndex); return; }
  float* buf = gbuf + warp * D;
  for (int which = 0; which < 2; ++which) {
    const TensorDesc& d = p.t[(tier == 1 ? 0 : 2) + which];
    T* out = reinterpret_cast<T*>(which ? p.out_v : p.out_k) + ((int64_t)s * p.T + tok) * D;
    for (int c = lane; c < D; c += 32) {
      int64_t e, gi;
      if (d.axis == GKV_AXIS_TOKEN) {
        e = ((int64_t)s * D + c) * d.n_pad + j;
        gi = ((int64_t)s * D + c) * d.groups_row + j / d.gs;
      } else {
        e = ((int64_t)s * n + j) * d.n_pad + c;
        gi = ((int64_t)s * n + j) * d.groups_row + c / d.gs;
      }
      const float v = decode_element(d, e, gi);
      if (d.rotation) buf[c] = v;
      else out[c] = Elem<T>::from_f32(v);
    }
    if (d.rotation) {
      __syncwarp();
      for (int h = 1; h < D; h <<= 1) {
        for (int q = lane; q < D / 2; q += 32) {
          const int i = (q / h) * 2 * h + (q % h);
          const float a = buf[i], b = buf[i + h];
          buf[i] = __fadd_rn(a, b);
          buf[i + h] = __fsub_rn(a, b);
        }
        __syncwarp();
      }
      for (int c = lane; c < D; c += 32) out[c] = hadamard_scale<T>(buf[c], p.had_div, p.had_inv);
      __syncwarp();
    }
  }
}

template <typename T>
__global__ void general_dequant_retained_kernel(const __grid_constant__ DequantParams p) {
  const int R = p.n_tier[0];
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)p.S * R * p.D) return;
  const int c = (int)(i % p.D);
  const int64_t rj = i / p.D;
  const int j = (int)(rj % R), s = (int)(rj / R);
  const int tok = p.idx[0][j];
  if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); return; }
  const int64_t o = ((int64_t)s * p.T + tok) * p.D + c;
  reinterpret_cast<T*>(p.out_k)[o] = reinterpret_cast<const T*>(p.ret_k)[i];
  reinterpret_cast<T*>(p.out_v)[o] = reinterpret_cast<const T*>(p.ret_v)[i];
}

// ---------------------------------------------------------------------------
// host-side launchers
// ---------------------------------------------------------------------------
template <typename T, int D, int TT>
static cudaError_t launch_dq_tile(const DequantParams& p, cudaStream_t st) {
  const size_t sm = dequant_tile_smem<T, D, TT>();
  auto kern = dequantize_tile_kernel<T, D, TT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.S * p.tiles_slice;
  if (blocks == 0) return cudaSuccess;
  kern<<<(unsigned)blocks, kThreads, sm, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_dq_tile_d(const DequantParams& p, cudaStream_t st) {
  if (p.D == 64) return p.tt == 64 ? launch_dq_tile<T, 64, 64>(p, st) : launch_dq_tile<T, 64, 128>(p, st);
  if (p.D == 128) {
    if (p.tt == 64) return launch_dq_tile<T, 128, 64>(p, st);
    if constexpr (sizeof(T) == 2) return launch_dq_tile<T, 128, 128>(p, st);
  }
  if constexpr (sizeof(T) == 2) {
    if (p.D == 256 && p.tt == 64) return launch_dq_tile<T, 256, 64>(p, st);
  }
  return cudaErrorInvalidConfiguration;
}

cudaError_t launch_dequantize_tiles(const DequantParams& p, int dtype, cudaStream_t st) {
  if (dtype == GKV_BF16) return launch_dq_tile_d<__nv_bfloat16>(p, st);
  if (dtype == GKV_F16) return launch_dq_tile_d<__half>(p, st);
  return launch_dq_tile_d<float>(p, st);
}

template <typename T>
static cudaError_t launch_dq_general_t(const DequantParams& p, int tier, cudaStream_t st) {
  const int64_t rows = (int64_t)p.S * p.n_tier[tier];
  if (rows == 0) return cudaSuccess;
  const size_t sm = 8 * (size_t)p.D * sizeof(float);
  cudaError_t e =
      cudaFuncSetAttribute(general_dequant_rows_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  general_dequant_rows_kernel<T><<<(unsigned)ceil_div(rows, 8), 256, sm, st>>>(p, tier);
  return cudaGetLastError();
}

cudaError_t launch_dequantize_general(const DequantParams& p, int dtype, int tier, cudaStream_t st) {
  if (dtype == GKV_BF16) return launch_dq_general_t<__nv_bfloat16>(p, tier, st);
  if (dtype == GKV_F16) return launch_dq_general_t<__half>(p, tier, st);
  return launch_dq_general_t<float>(p, tier, st);
}

cudaError_t launch_dequantize_retained_general(const DequantParams& p, int dtype, cudaStream_t st) {
  const int64_t total = (int64_t)p.S * p.n_tier[0] * p.D;
  if (total == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)ceil_div(total, 256);
  if (dtype == GKV_BF16) general_dequant_retained_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p);
  else if (dtype == GKV_F16) general_dequant_retained_kernel<__half><<<blocks, 256, 0, st>>>(p);
  else general_dequant_retained_kernel<float><<<blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace gkv
