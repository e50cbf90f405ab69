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

// two codes at once: (enc ^ xor) + off, times the scale, in packed fp32
__device__ __forceinline__ uint64_t decode2(uint32_t e0, uint32_t e1, const Decoder& dc) {
  const uint64_t q = sub2(pk2(__uint_as_float(0x4B000000u | (e0 ^ dc.xor_mask)),
                              __uint_as_float(0x4B000000u | (e1 ^ dc.xor_mask))),
                          pk2(dc.base, dc.base));
  return mul2(q, pk2(dc.scale, dc.scale));
}

__device__ __forceinline__ int load_zp(const TensorDesc& d, int64_t gi) {
  return d.quantizer == GKV_AFFINE ? (int)d.zps[gi] : 0;
}

// Output of one decoded row (lane holds D/32 consecutive channels): optional
// inverse rotation across the warp, cast to T, one vector store per lane.
// Cross-lane butterfly stages compute o + sign * v with one fused multiply-add:
// sign = +1 gives v + o, sign = -1 gives o - v, each rounded once as the
// reference's add / subtract.
template <typename T, int D, bool ROT>
__device__ __forceinline__ void emit_row(float (&v)[D / 32], float div, float inv, T* dst) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  if constexpr (ROT) fwht_warp<EPL>(v);
  constexpr int NB = EPL * (int)sizeof(T);
  constexpr int NW = NB / 4;
  uint32_t w[NW];
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < EPL; ++i) w[i] = __float_as_uint(ROT ? __fdiv_rn(v[i], div) : v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < EPL; i += 2) {
      uint32_t lo, hi;
      if constexpr (ROT) {
        lo = tbits(hadamard_scale<T>(v[i], div, inv));
        hi = tbits(hadamard_scale<T>(v[i + 1], div, inv));
        w[i / 2] = lo | (hi << 16);
      } else if constexpr (Elem<T>::kTag == GKV_BF16) {
        const __nv_bfloat162 p = __floats2bfloat162_rn(v[i], v[i + 1]);
        w[i / 2] = *reinterpret_cast<const uint32_t*>(&p);
      } else {
        const __half2 p = __floats2half2_rn(v[i], v[i + 1]);
        w[i / 2] = *reinterpret_cast<const uint32_t*>(&p);
      }
    }
  }
  store_bytes<NB>(reinterpret_cast<uint8_t*>(dst + lane * EPL), w);
}


// 32 codes of a run (SB bits each) as fp32 bit patterns 2^23 + code
template <int SB>
__device__ __forceinline__ void run_codes(const uint32_t (&w)[SB], uint32_t (&c)[kRun]) {
#pragma unroll
  for (int q = 0; q < SB; ++q) {
    uint32_t t[32 / SB];
    word_codes<SB>(w[q], t);
#pragma unroll
    for (int i = 0; i < 32 / SB; ++i) c[q * (32 / SB) + i] = t[i];
  }
}

template <int SB>
__device__ __forceinline__ void load_run(const uint8_t* p, uint32_t (&w)[SB]) {
  if constexpr (SB == 2) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    w[0] = t.x; w[1] = t.y;
  } else if constexpr (SB == 4) {
    const uint4 t = *reinterpret_cast<const uint4*>(p);
    w[0] = t.x; w[1] = t.y; w[2] = t.z; w[3] = t.w;
  } else {
    const uint4 t0 = reinterpret_cast<const uint4*>(p)[0], t1 = reinterpret_cast<const uint4*>(p)[1];
    w[0] = t0.x; w[1] = t0.y; w[2] = t0.z; w[3] = t0.w; w[4] = t1.x; w[5] = t1.y; w[6] = t1.z; w[7] = t1.w;
  }
}

// decoded values of a run: ((2^23 + code) ^ xor) - base, times the scale, in packed pairs
__device__ __forceinline__ void decode_run(const uint32_t (&c)[kRun], const Decoder& dc, float (&v)[kRun]) {
  const uint64_t base2 = pk2(dc.base, dc.base), sc2 = pk2(dc.scale, dc.scale);
#pragma unroll
  for (int i = 0; i < kRun; i += 2) {
    const uint64_t q = sub2(pk2(__uint_as_float(c[i] ^ dc.xor_mask), __uint_as_float(c[i + 1] ^ dc.xor_mask)), base2);
    const uint64_t r = mul2(q, sc2);
    v[i] = lo2(r);
    v[i + 1] = hi2(r);
  }
}

// pack two fp32 values into one 32-bit word of T (round to nearest even)
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  if constexpr (Elem<T>::kTag == GKV_BF16) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&p);
  } else {
    const __half2 p = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&p);
  }
}

// Channel-axis tensor (values by default): item = (tier row, run of 32 channels),
// the runs of a row in adjacent lanes (the Hadamard rotation crosses them with
// shuffles).  Codes, scale and zero point are loaded once per run, decoded in
// registers and stored with 16-byte vector stores at the row's output position.
template <typename T, int D, int TT, int SB, bool ROT>
__device__ void dequant_channel_half(const DequantParams& p, const TensorDesc& d, T* out, const int* tok, int s,
                                     int j0, int rows) {
  constexpr int RPR = D / kRun;
  constexpr int ITEMS = TT * RPR;
  constexpr int ITER = (ITEMS + 127) / 128;
  const int ht = threadIdx.x & 127;
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int itn = 0; itn < ITER; ++itn) {
    const int item = ht + itn * 128;
    const int r = item / RPR, run = item % RPR;
    const bool act = item < ITEMS && r < rows;
    uint32_t w[SB];
#pragma unroll
    for (int q = 0; q < SB; ++q) w[q] = 0;
    float scale = 0.f;
    int zp = 0;
    if (act) {
      const int64_t row = (int64_t)s * d.n + j0 + r;
      load_run<SB>(d.codes + ((row * d.n_pad + run * kRun) * SB) / 8, w);
      const int64_t gi = row * d.groups_row + ((run * kRun) >> d.log2gs);
      scale = load_scale(d.scales, gi, d.scale_dtype);
      zp = load_zp(d, gi);
    }
    uint32_t c[kRun];
    run_codes<SB>(w, c);
    float v[kRun];
    decode_run(c, make_decoder(d, scale, zp), v);
    if constexpr (ROT) {
      // in-thread stages h = 1 .. 16, then across the RPR lanes of the row
#pragma unroll
      for (int h = 1; h < kRun; h <<= 1) {
#pragma unroll
        for (int i = 0; i < kRun; i += 2 * h) {
#pragma unroll
          for (int j = 0; j < h; ++j) {
            const float a = v[i + j], bb = v[i + j + h];
            v[i + j] = __fadd_rn(a, bb);
            v[i + j + h] = __fsub_rn(a, bb);
          }
        }
      }
#pragma unroll
      for (int m = 1; m < RPR; m <<= 1) {
        const float sg = (lane & m) ? -1.f : 1.f;
        const uint64_t sg2 = pk2(sg, sg);
#pragma unroll
        for (int i = 0; i < kRun; i += 2) {
          const float o0 = __shfl_xor_sync(0xFFFFFFFFu, v[i], m);
          const float o1 = __shfl_xor_sync(0xFFFFFFFFu, v[i + 1], m);
          const uint64_t rr = fma2(sg2, pk2(v[i], v[i + 1]), pk2(o0, o1));
          v[i] = lo2(rr);
          v[i + 1] = hi2(rr);
        }
      }
    }
    if (act && tok[r] >= 0) {
      T* dst = out + (int64_t)tok[r] * D + run * kRun;
      if constexpr (sizeof(T) == 4) {
#pragma unroll
        for (int q = 0; q < kRun / 4; ++q) {
          float o[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) o[u] = ROT ? __fdiv_rn(v[4 * q + u], p.had_div) : v[4 * q + u];
          reinterpret_cast<uint4*>(dst)[q] =
              make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]), __float_as_uint(o[3]));
        }
      } else {
#pragma unroll
        for (int q = 0; q < kRun / 8; ++q) {
          uint32_t o[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float a = v[8 * q + 2 * u], bb = v[8 * q + 2 * u + 1];
            if constexpr (ROT)
              o[u] = tbits(hadamard_scale<T>(a, p.had_div, p.had_inv)) |
                     (tbits(hadamard_scale<T>(bb, p.had_div, p.had_inv)) << 16);
            else
              o[u] = pack_pair<T>(a, bb);
          }
          reinterpret_cast<uint4*>(dst)[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
}

// Token-axis tensor (keys by default): item = (32-bit column word, run of 32 rows);
// the decoded values are written into the half's shared tile [TT][D + pad] of T,
// then whole rows leave with 16-byte vector stores.  (Rotated token-axis tensors
// take the general path.)
template <typename T, int D, int TT, int SB>
__device__ void dequant_token_half(const DequantParams& p, const TensorDesc& d, T* out, const int* tok, int s, int j0,
                                   int rows, T* tile, int half) {
  constexpr int CPW = 4 / (int)sizeof(T);
  constexpr int W = D / CPW;
  constexpr int NRUN = TT / kRun;
  constexpr int ITEMS = W * NRUN;
  constexpr int ITER = (ITEMS + 127) / 128;
  constexpr int TP = D + 16 / (int)sizeof(T);  // tile pitch (elements)
  const int ht = threadIdx.x & 127;
#pragma unroll 1
  for (int itn = 0; itn < ITER; ++itn) {
    const int item = ht + itn * 128;
    if (item >= ITEMS) break;
    const int w = item % W, run = item / W;
    const int tk = j0 + run * kRun;
    if (tk >= d.n_pad) continue;
    float v[CPW][kRun];
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int64_t crow = (int64_t)s * D + w * CPW + c;
      uint32_t cw[SB];
      load_run<SB>(d.codes + ((crow * d.n_pad + tk) * SB) / 8, cw);
      const int64_t gi = crow * d.groups_row + (tk >> d.log2gs);
      uint32_t codes[kRun];
      run_codes<SB>(cw, codes);
      decode_run(codes, make_decoder(d, load_scale(d.scales, gi, d.scale_dtype), load_zp(d, gi)), v[c]);
    }
    uint32_t* col = reinterpret_cast<uint32_t*>(tile + (run * kRun) * TP) + w;
#pragma unroll
    for (int i = 0; i < kRun; ++i) {
      if constexpr (CPW == 2) col[i * (TP / 2)] = pack_pair<T>(v[0][i], v[1][i]);
      else col[i * TP] = __float_as_uint(v[0][i]);
    }
  }
  bar_half(half);
  constexpr int CPR = D * (int)sizeof(T) / 16;  // 16-byte chunks per row
  for (int e = ht; e < rows * CPR; e += 128) {
    const int r = e / CPR, c = e - r * CPR;
    if (tok[r] < 0) continue;
    reinterpret_cast<uint4*>(out + (int64_t)tok[r] * D)[c] = reinterpret_cast<const uint4*>(tile + r * TP)[c];
  }
}

template <typename T, int D, int TT, bool ROT>
__device__ __forceinline__ void dequant_half_rot(const DequantParams& p, const TensorDesc& d, T* out, const int* tok,
                                                 int s, int j0, int rows, T* tile, int half) {
  if (d.axis == GKV_AXIS_TOKEN) {
    if constexpr (!ROT) {
      if (d.sbits == 4) dequant_token_half<T, D, TT, 4>(p, d, out, tok, s, j0, rows, tile, half);
      else if (d.sbits == 2) dequant_token_half<T, D, TT, 2>(p, d, out, tok, s, j0, rows, tile, half);
      else dequant_token_half<T, D, TT, 8>(p, d, out, tok, s, j0, rows, tile, half);
    }
  } else {
    if (d.sbits == 4) dequant_channel_half<T, D, TT, 4, ROT>(p, d, out, tok, s, j0, rows);
    else if (d.sbits == 2) dequant_channel_half<T, D, TT, 2, ROT>(p, d, out, tok, s, j0, rows);
    else dequant_channel_half<T, D, TT, 8, ROT>(p, d, out, tok, s, j0, rows);
  }
}

template <typename T, int D, int TT>
constexpr size_t dequant_tile_smem() {
  return 2 * (size_t)TT * (D + 16 / sizeof(T)) * sizeof(T) + (size_t)TT * sizeof(int);
}

// One block per tile: retained tiles scatter their rows; standard / cold tiles load
// the tile's output positions once, then warps 0-3 decode K and warps 4-7 decode V.
template <typename T, int D, int TT>
__global__ void __launch_bounds__(kThreads, 3) dequantize_tile_kernel(const __grid_constant__ DequantParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
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
  const int* idx = p.idx[tier];
  const int j0 = k * TT;
  const int rows = min(TT, p.n_tier[tier] - j0);
  constexpr int TP = D + 16 / (int)sizeof(T);
  T* tiles = reinterpret_cast<T*>(smem);
  int* tok = reinterpret_cast<int*>(smem + 2 * (size_t)TT * TP * sizeof(T));
  for (int r = threadIdx.x; r < TT; r += kThreads) {
    int t = -1;
    if (r < rows) {
      t = idx[j0 + r];
      if ((unsigned)t >= (unsigned)p.T) { raise_error(kErrBadIndex); t = -1; }
    }
    tok[r] = t;
  }
  __syncthreads();
  const int half = threadIdx.x >> 7;
  const TensorDesc& d = p.t[(tier == 1 ? GKV_STD_K : GKV_COLD_K) + half];
  T* out = half ? ov : ok;
  if (d.rotation) dequant_half_rot<T, D, TT, true>(p, d, out, tok, s, j0, rows, tiles + half * TT * TP, half);
  else dequant_half_rot<T, D, TT, false>(p, d, out, tok, s, j0, rows, tiles + half * TT * TP, half);
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
  if (p.D == 128) return p.tt == 64 ? launch_dq_tile<T, 128, 64>(p, st) : launch_dq_tile<T, 128, 128>(p, st);
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
