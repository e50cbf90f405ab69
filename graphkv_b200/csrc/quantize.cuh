// Quantize + pack kernels (core.py:647-772, 848-910, 945-956, 979-990).
//
// Fast path: one block per tile of TT consecutive tier rows of one slice.  Warp 0
// gathers the K and V rows of the tile into shared memory with bulk async copies
// (one row per copy, completion on an mbarrier), rows are rotated in place when the
// tensor uses the Hadamard rotation, then each tensor is grouped along its axis,
// scaled and packed straight to HBM.  Retained rows are copied by tiles of the same
// launch.
//
// General path: any geometry the tiles do not cover (group sizes that are not
// powers of two, padded head dims, tiny tiers, unaligned inputs): one thread per
// group computes the scale, one thread per output byte packs the codes.
#pragma once

#include "gkv_params.cuh"

namespace gkv {

// ---------------------------------------------------------------------------
// element access
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void unpack_word(uint32_t w, float (&f)[4 / sizeof(T)]) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(w);
  } else if constexpr (Elem<T>::kTag == GKV_BF16) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xFFFF0000u);
  } else {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w));
    f[0] = t.x;
    f[1] = t.y;
  }
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename T, int D>
struct RowGeom {
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kPitch = D + 16 / (int)sizeof(T);  // +16 B per row spreads rows over banks
  static constexpr int kVec = 16 / (int)sizeof(T);
  static constexpr int kChunks = D / kVec;
  static constexpr int kWords = kRowBytes / 4;
  static constexpr int kSegs = kThreads / kWords;         // token-axis segments per tile
};

// ---------------------------------------------------------------------------
// fast path pieces
// ---------------------------------------------------------------------------
template <typename T, int D>
__device__ void copy_retained_tile(const QuantParams& p, const T* kb, const T* vb, int64_t kst, int64_t vst,
                                   int gslice, int tile) {
  using G = RowGeom<T, D>;
  const int R = p.n_tier[0];
  const int j0 = tile * kRetTile;
  const int rows = min(kRetTile, R - j0);
  T* rk = reinterpret_cast<T*>(p.ret_k) + ((int64_t)gslice * R + j0) * D;
  T* rv = reinterpret_cast<T*>(p.ret_v) + ((int64_t)gslice * R + j0) * D;
  for (int e = threadIdx.x; e < rows * G::kChunks; e += kThreads) {
    const int r = e / G::kChunks, c = e - r * G::kChunks;
    int tok = p.idx[0][j0 + r];
    if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); tok = 0; }
    const uint4 a = ldg_stream(kb + tok * kst + c * G::kVec);
    const uint4 b = ldg_stream(vb + tok * vst + c * G::kVec);
    *reinterpret_cast<uint4*>(rk + r * D + c * G::kVec) = a;
    *reinterpret_cast<uint4*>(rv + r * D + c * G::kVec) = b;
  }
}

// Hadamard rotation of `rows` rows held in shared memory, one warp per row.
// Butterfly stages run in the reference order h = 1, 2, 4, ... (core.py:950-955).
template <typename T, int D>
__device__ void rotate_rows_smem(T* sx, int rows, float div, float inv) {
  using G = RowGeom<T, D>;
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = warp; r < rows; r += kThreads / 32) {
    T* row = sx + r * G::kPitch + lane * EPL;
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = Elem<T>::to_f32(row[i]);
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
#pragma unroll
    for (int i = 0; i < EPL; ++i) row[i] = hadamard_scale<T>(v[i], div, inv);
  }
}

// Token-axis groups (keys by default): groups of gs consecutive tier rows of one
// channel.  Thread (word w, segment seg) holds SEG rows of 32-bit words.
template <typename T, int D, int TT, int SB, bool AFF>
__device__ void quant_token_tile(const TensorDesc& d, const T* sx, int gslice, int j0, float* red) {
  using G = RowGeom<T, D>;
  constexpr int W = G::kWords;
  constexpr int SEG = TT / G::kSegs;
  constexpr int CPW = 4 / (int)sizeof(T);
  const int tid = threadIdx.x;
  const int w = tid % W, seg = tid / W;

  uint32_t x[SEG];
#pragma unroll
  for (int i = 0; i < SEG; ++i) x[i] = reinterpret_cast<const uint32_t*>(sx + (seg * SEG + i) * G::kPitch)[w];

  float mn[CPW], mx[CPW];
#pragma unroll
  for (int c = 0; c < CPW; ++c) { mn[c] = __int_as_float(0x7f800000); mx[c] = -__int_as_float(0x7f800000); }
#pragma unroll
  for (int i = 0; i < SEG; ++i) {
    float f[CPW];
    unpack_word<T>(x[i], f);
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      if (AFF) { mn[c] = fminf(mn[c], f[c]); mx[c] = fmaxf(mx[c], f[c]); }
      else { mx[c] = fmaxf(mx[c], fabsf(f[c])); }
    }
  }
  const int spg = d.gs / SEG;  // segments per group (host guarantees gs >= SEG, TT % gs == 0)
  if (spg > 1) {
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int ch = w * CPW + c;
      red[(seg * D + ch) * 2 + 0] = mn[c];
      red[(seg * D + ch) * 2 + 1] = mx[c];
    }
    __syncthreads();
    const int s0 = (seg / spg) * spg;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int ch = w * CPW + c;
      for (int q = 0; q < spg; ++q) {
        if (AFF) mn[c] = fminf(mn[c], red[((s0 + q) * D + ch) * 2 + 0]);
        mx[c] = fmaxf(mx[c], red[((s0 + q) * D + ch) * 2 + 1]);
      }
    }
    __syncthreads();
  }
  const int tok0 = j0 + (seg / spg) * d.gs;  // first tier row of this thread's group
  if (tok0 >= d.n_pad) return;
  const int g = tok0 >> d.log2gs;
#pragma unroll
  for (int c = 0; c < CPW; ++c) {
    const int ch = w * CPW + c;
    const GroupCoder cd = AFF ? make_affine(mn[c], mx[c], d.bits) : make_symmetric(mx[c], d.bits, d.packed != 0);
    if (seg % spg == 0) {
      const int64_t gi = ((int64_t)gslice * D + ch) * d.groups_row + g;
      store_scale(d.scales, gi, d.scale_dtype, cd.scale);
      if (AFF) d.zps[gi] = (uint8_t)cd.zpi;
    }
    constexpr int NW = (SEG * SB + 31) / 32;
    uint32_t out[NW];
#pragma unroll
    for (int q = 0; q < NW; ++q) out[q] = 0;
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      float f[CPW];
      unpack_word<T>(x[i], f);
      const uint32_t code = code_of(f[c], cd) & ((1u << SB) - 1u);
      out[(i * SB) / 32] |= code << ((i * SB) % 32);
    }
    const int64_t e0 = ((int64_t)gslice * D + ch) * d.n_pad + j0 + seg * SEG;
    store_bytes<SEG * SB / 8>(d.codes + (e0 * SB) / 8, out);
  }
}

// Channel-axis groups (values by default): groups of gs consecutive channels of one
// token.  Thread per 16-byte chunk; the gs / VEC chunks of a group are adjacent lanes.
template <typename T, int D, int TT, int SB, bool AFF>
__device__ void quant_channel_tile(const TensorDesc& d, const T* sx, int gslice, int j0, int rows) {
  using G = RowGeom<T, D>;
  constexpr int VEC = G::kVec;
  constexpr int CPR = G::kChunks;
  constexpr int EPW = 4 / (int)sizeof(T);
  const int cpg = d.gs / VEC;
  for (int it = threadIdx.x; it < TT * CPR; it += kThreads) {
    const int r = it / CPR, c = it - r * CPR;
    const uint4 raw = *reinterpret_cast<const uint4*>(sx + r * G::kPitch + c * VEC);
    const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
    float v[VEC];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float f[EPW];
      unpack_word<T>(wv[q], f);
#pragma unroll
      for (int u = 0; u < EPW; ++u) v[q * EPW + u] = f[u];
    }
    float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      if (AFF) { mn = fminf(mn, v[i]); mx = fmaxf(mx, v[i]); }
      else mx = fmaxf(mx, fabsf(v[i]));
    }
    for (int m = 1; m < cpg; m <<= 1) {
      if (AFF) mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, m));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, m));
    }
    if (r < rows) {
      const GroupCoder cd = AFF ? make_affine(mn, mx, d.bits) : make_symmetric(mx, d.bits, d.packed != 0);
      const int64_t row = (int64_t)gslice * d.n + j0 + r;
      if ((c & (cpg - 1)) == 0) {
        const int64_t gi = row * d.groups_row + c / cpg;
        store_scale(d.scales, gi, d.scale_dtype, cd.scale);
        if (AFF) d.zps[gi] = (uint8_t)cd.zpi;
      }
      constexpr int NW = (VEC * SB + 31) / 32;
      uint32_t out[NW];
#pragma unroll
      for (int q = 0; q < NW; ++q) out[q] = 0;
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const uint32_t code = code_of(v[i], cd) & ((1u << SB) - 1u);
        out[(i * SB) / 32] |= code << ((i * SB) % 32);
      }
      const int64_t e0 = row * d.n_pad + c * VEC;
      store_bytes<VEC * SB / 8>(d.codes + (e0 * SB) / 8, out);
    }
  }
}

template <typename T, int D, int TT, int SB>
__device__ __forceinline__ void quant_tensor_sb(const TensorDesc& d, const T* sx, int gslice, int j0, int rows,
                                                float* red) {
  const bool aff = d.quantizer == GKV_AFFINE;
  if (d.axis == GKV_AXIS_TOKEN) {
    if (aff) quant_token_tile<T, D, TT, SB, true>(d, sx, gslice, j0, red);
    else quant_token_tile<T, D, TT, SB, false>(d, sx, gslice, j0, red);
  } else {
    if (aff) quant_channel_tile<T, D, TT, SB, true>(d, sx, gslice, j0, rows);
    else quant_channel_tile<T, D, TT, SB, false>(d, sx, gslice, j0, rows);
  }
}

template <typename T, int D, int TT>
__device__ __forceinline__ void quant_tensor(const TensorDesc& d, const T* sx, int gslice, int j0, int rows,
                                             float* red) {
  if (d.sbits == 4) quant_tensor_sb<T, D, TT, 4>(d, sx, gslice, j0, rows, red);
  else if (d.sbits == 2) quant_tensor_sb<T, D, TT, 2>(d, sx, gslice, j0, rows, red);
  else quant_tensor_sb<T, D, TT, 8>(d, sx, gslice, j0, rows, red);
}

template <typename T, int D, int TT>
constexpr size_t quant_tile_smem() {
  using G = RowGeom<T, D>;
  return 2 * (size_t)TT * G::kPitch * sizeof(T) + (size_t)G::kSegs * D * 2 * sizeof(float) + 16;
}

template <typename T, int D, int TT>
__global__ void __launch_bounds__(kThreads) quantize_tile_kernel(const __grid_constant__ QuantParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  using G = RowGeom<T, D>;
  const int s = blockIdx.x / p.tiles_slice;
  int k = blockIdx.x - s * p.tiles_slice;
  const LayerDesc& L = p.layers[find_layer(p, s)];
  const int local = s - L.slice_begin;
  const int b = local / L.heads, h = local - b * L.heads;
  const T* kb = reinterpret_cast<const T*>(L.k) + b * L.ks[0] + h * L.ks[1];
  const T* vb = reinterpret_cast<const T*>(L.v) + b * L.vs[0] + h * L.vs[1];
  const int gslice = p.slice_offset + s;

  if (k < p.tiles[0]) {
    copy_retained_tile<T, D>(p, kb, vb, L.ks[2], L.vs[2], gslice, k);
    return;
  }
  k -= p.tiles[0];
  int tier = 1;
  if (k >= p.tiles[1]) { k -= p.tiles[1]; tier = 2; }
  const TensorDesc& dk = p.t[tier == 1 ? GKV_STD_K : GKV_COLD_K];
  const TensorDesc& dv = p.t[tier == 1 ? GKV_STD_V : GKV_COLD_V];
  const int* idx = p.idx[tier];
  const int n = p.n_tier[tier];
  const int j0 = k * TT;
  const int rows = min(TT, n - j0);

  T* sk = reinterpret_cast<T*>(smem);
  T* sv = sk + TT * G::kPitch;
  float* red = reinterpret_cast<float*>(sv + TT * G::kPitch);
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + G::kSegs * D * 2);

  if (threadIdx.x == 0) mbar_init(bar, 1);
  __syncthreads();
  if (threadIdx.x < 32) {
    if (threadIdx.x == 0) mbar_arrive_expect_tx(bar, (uint32_t)(rows * 2 * G::kRowBytes));
    __syncwarp();
    for (int r = threadIdx.x; r < rows; r += 32) {
      int tok = idx[j0 + r];
      if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); tok = 0; }
      bulk_load(sk + r * G::kPitch, kb + tok * L.ks[2], G::kRowBytes, bar);
      bulk_load(sv + r * G::kPitch, vb + tok * L.vs[2], G::kRowBytes, bar);
    }
  }
  // rows past the end of the tier are zero: token-axis groups quantize them as padding
  for (int e = threadIdx.x; e < (TT - rows) * G::kChunks; e += kThreads) {
    const int r = rows + e / G::kChunks, c = e % G::kChunks;
    *reinterpret_cast<uint4*>(sk + r * G::kPitch + c * G::kVec) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(sv + r * G::kPitch + c * G::kVec) = make_uint4(0, 0, 0, 0);
  }
  if (!block_wait(bar, 0)) return;

  if (dk.rotation) rotate_rows_smem<T, D>(sk, rows, p.had_div, p.had_inv);
  if (dv.rotation) rotate_rows_smem<T, D>(sv, rows, p.had_div, p.had_inv);
  if (dk.rotation | dv.rotation) __syncthreads();

  quant_tensor<T, D, TT>(dk, sk, gslice, j0, rows, red);
  quant_tensor<T, D, TT>(dv, sv, gslice, j0, rows, red);
}

// ---------------------------------------------------------------------------
// general path
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float input_value(const QuantParams& p, bool is_v, int s, int tok, int c) {
  const LayerDesc& L = p.layers[find_layer(p, s)];
  const int local = s - L.slice_begin;
  const int b = local / L.heads, h = local - b * L.heads;
  const T* base = reinterpret_cast<const T*>(is_v ? L.v : L.k);
  const int64_t* st = is_v ? L.vs : L.ks;
  return Elem<T>::to_f32(base[b * st[0] + h * st[1] + (int64_t)tok * st[2] + c]);
}

__device__ __forceinline__ int checked_token(const QuantParams& p, int tier, int j) {
  int tok = p.idx[tier][j];
  if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); tok = 0; }
  return tok;
}

// value of tier row j, channel c of tensor ti in slice s (rotated copy when rotating)
template <typename T>
__device__ __forceinline__ float tier_value(const QuantParams& p, int ti, int tier, int s, int j, int c) {
  const TensorDesc& d = p.t[ti];
  if (d.rotation) {
    const int gslice = p.slice_offset + s;
    return Elem<T>::to_f32(reinterpret_cast<const T*>(d.rot)[((int64_t)gslice * d.n + j) * p.D + c]);
  }
  return input_value<T>(p, (ti & 1) != 0, s, checked_token(p, tier, j), c);
}

// one warp per tier row: rotated rows into the workspace (D a power of two <= 1024)
template <typename T>
__global__ void __launch_bounds__(256) general_rotate_kernel(const __grid_constant__ QuantParams p, int ti, int tier) {
  extern __shared__ float rbuf[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  const TensorDesc& d = p.t[ti];
  if (row >= (int64_t)p.S * d.n) return;
  const int s = (int)(row / d.n), j = (int)(row % d.n);
  const int D = p.D;
  float* buf = rbuf + warp * D;
  const int tok = checked_token(p, tier, j);
  for (int c = lane; c < D; c += 32) buf[c] = input_value<T>(p, (ti & 1) != 0, s, tok, c);
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
  T* out = reinterpret_cast<T*>(d.rot) + (((int64_t)(p.slice_offset + s)) * d.n + j) * D;
  for (int c = lane; c < D; c += 32) out[c] = hadamard_scale<T>(buf[c], p.had_div, p.had_inv);
}

// one thread per group: coding scale (fp32, workspace), stored scale and zero point
template <typename T>
__global__ void general_stats_kernel(const __grid_constant__ QuantParams p, int ti, int tier) {
  const TensorDesc& d = p.t[ti];
  const int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gi >= (int64_t)p.S * d.groups_slice) return;
  const int s = (int)(gi / d.groups_slice);
  const int64_t lg = gi - (int64_t)s * d.groups_slice;
  const int a = (int)(lg / d.groups_row), g = (int)(lg % d.groups_row);
  float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000), amax = 0.f;
  for (int u = 0; u < d.gs; ++u) {
    const int e = g * d.gs + u;  // position along the grouped axis (may be padding)
    float x = 0.f;
    if (d.axis == GKV_AXIS_TOKEN) {
      if (e < d.n) x = tier_value<T>(p, ti, tier, s, e, a);
    } else {
      if (e < p.D) x = tier_value<T>(p, ti, tier, s, a, e);
    }
    mn = fminf(mn, x);
    mx = fmaxf(mx, x);
    amax = fmaxf(amax, fabsf(x));
  }
  const GroupCoder cd = d.quantizer == GKV_AFFINE ? make_affine(mn, mx, d.bits)
                                                  : make_symmetric(amax, d.bits, d.packed != 0);
  const int64_t ggi = (int64_t)p.slice_offset * d.groups_slice + gi;
  d.scale32[ggi] = cd.scale;
  store_scale(d.scales, ggi, d.scale_dtype, cd.scale);
  if (d.quantizer == GKV_AFFINE) d.zps[ggi] = (uint8_t)cd.zpi;
}

__device__ __forceinline__ GroupCoder coder_from(const TensorDesc& d, float scale, int zp) {
  GroupCoder c;
  c.scale = scale;
  c.inv = __frcp_rn(scale);
  if (d.quantizer == GKV_AFFINE) {
    c.lo = 0.f;
    c.hi = (float)((1 << d.bits) - 1);
    c.zpi = zp;
    c.zp = (float)zp;
    c.magic = kMagic;
  } else {
    const int qmin = -(1 << (d.bits - 1));
    c.lo = (float)qmin;
    c.hi = (float)((1 << (d.bits - 1)) - 1);
    c.zpi = 0;
    c.zp = 0.f;
    c.magic = kMagic + (d.packed ? (float)(-qmin) : 0.f);
  }
  return c;
}

// one thread per output byte of this launch's part of the code stream
template <typename T>
__global__ void general_pack_kernel(const __grid_constant__ QuantParams p, int ti, int tier) {
  const TensorDesc& d = p.t[ti];
  const int vpb = 8 / d.sbits;
  const int64_t E = (int64_t)p.S * d.elems_slice;
  const int64_t nbytes = (E * d.sbits + 7) / 8;
  const int64_t byte = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (byte >= nbytes) return;
  const uint32_t mask = (1u << d.sbits) - 1u;
  uint32_t acc = 0;
  for (int i = 0; i < vpb; ++i) {
    const int64_t e = byte * vpb + i;
    if (e >= E) break;
    const int s = (int)(e / d.elems_slice);
    const int64_t le = e - (int64_t)s * d.elems_slice;
    const int a = (int)(le / d.n_pad), b = (int)(le % d.n_pad);
    float x = 0.f;
    if (d.axis == GKV_AXIS_TOKEN) {  // a = channel, b = tier row
      if (b < d.n) x = tier_value<T>(p, ti, tier, s, b, a);
    } else {  // a = tier row, b = channel
      if (b < p.D) x = tier_value<T>(p, ti, tier, s, a, b);
    }
    const int64_t lg = (int64_t)a * d.groups_row + b / d.gs;
    const int64_t ggi = ((int64_t)p.slice_offset + s) * d.groups_slice + lg;
    const GroupCoder cd = coder_from(d, d.scale32[ggi], d.quantizer == GKV_AFFINE ? (int)d.zps[ggi] : 0);
    acc |= (code_of(x, cd) & mask) << (i * d.sbits);
  }
  d.codes[(int64_t)p.slice_offset * d.elems_slice * d.sbits / 8 + byte] = (uint8_t)acc;
}

template <typename T>
__global__ void general_retained_kernel(const __grid_constant__ QuantParams p) {
  const int R = p.n_tier[0];
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)p.S * R * p.D;
  if (i >= total) return;
  const int c = (int)(i % p.D);
  const int64_t rj = i / p.D;
  const int j = (int)(rj % R), s = (int)(rj / R);
  const int tok = checked_token(p, 0, j);
  const LayerDesc& L = p.layers[find_layer(p, s)];
  const int local = s - L.slice_begin;
  const int b = local / L.heads, h = local - b * L.heads;
  const int64_t o = (((int64_t)p.slice_offset + s) * R + j) * p.D + c;
  reinterpret_cast<T*>(p.ret_k)[o] =
      reinterpret_cast<const T*>(L.k)[b * L.ks[0] + h * L.ks[1] + (int64_t)tok * L.ks[2] + c];
  reinterpret_cast<T*>(p.ret_v)[o] =
      reinterpret_cast<const T*>(L.v)[b * L.vs[0] + h * L.vs[1] + (int64_t)tok * L.vs[2] + c];
}

// ---------------------------------------------------------------------------
// host-side launchers (called from capi.cu)
// ---------------------------------------------------------------------------
template <typename T, int D, int TT>
static cudaError_t launch_tile(const QuantParams& p, cudaStream_t st) {
  const size_t sm = quant_tile_smem<T, D, TT>();
  auto kern = quantize_tile_kernel<T, D, TT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.S * p.tiles_slice;
  if (blocks == 0) return cudaSuccess;
  kern<<<(unsigned)blocks, kThreads, sm, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_tile_d(const QuantParams& p, cudaStream_t st) {
  if (p.D == 64) return p.tt == 64 ? launch_tile<T, 64, 64>(p, st) : launch_tile<T, 64, 128>(p, st);
  if (p.D == 128) {
    if (p.tt == 64) return launch_tile<T, 128, 64>(p, st);
    if constexpr (sizeof(T) == 2) return launch_tile<T, 128, 128>(p, st);
  }
  if constexpr (sizeof(T) == 2) {
    if (p.D == 256 && p.tt == 64) return launch_tile<T, 256, 64>(p, st);
  }
  return cudaErrorInvalidConfiguration;
}

cudaError_t launch_quantize_tiles(const QuantParams& p, int dtype, cudaStream_t st) {
  if (dtype == GKV_BF16) return launch_tile_d<__nv_bfloat16>(p, st);
  if (dtype == GKV_F16) return launch_tile_d<__half>(p, st);
  return launch_tile_d<float>(p, st);
}

template <typename T>
static cudaError_t launch_general_t(const QuantParams& p, int ti, int tier, cudaStream_t st) {
  const TensorDesc& d = p.t[ti];
  cudaError_t e;
  if (d.rotation) {
    const int64_t rows = (int64_t)p.S * d.n;
    const size_t sm = 8 * (size_t)p.D * sizeof(float);
    e = cudaFuncSetAttribute(general_rotate_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    general_rotate_kernel<T><<<(unsigned)ceil_div(rows, 8), 256, sm, st>>>(p, ti, tier);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const int64_t groups = (int64_t)p.S * d.groups_slice;
  general_stats_kernel<T><<<(unsigned)ceil_div(groups, 128), 128, 0, st>>>(p, ti, tier);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const int64_t nbytes = ((int64_t)p.S * d.elems_slice * d.sbits + 7) / 8;
  general_pack_kernel<T><<<(unsigned)ceil_div(nbytes, 256), 256, 0, st>>>(p, ti, tier);
  return cudaGetLastError();
}

cudaError_t launch_quantize_general(const QuantParams& p, int dtype, int ti, int tier, cudaStream_t st) {
  if (dtype == GKV_BF16) return launch_general_t<__nv_bfloat16>(p, ti, tier, st);
  if (dtype == GKV_F16) return launch_general_t<__half>(p, ti, tier, st);
  return launch_general_t<float>(p, ti, tier, st);
}

cudaError_t launch_retained_general(const QuantParams& p, int dtype, cudaStream_t st) {
  const int64_t total = (int64_t)p.S * p.n_tier[0] * p.D;
  if (total == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)ceil_div(total, 256);
  if (dtype == GKV_BF16) general_retained_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p);
  else if (dtype == GKV_F16) general_retained_kernel<__half><<<blocks, 256, 0, st>>>(p);
  else general_retained_kernel<float><<<blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace gkv
