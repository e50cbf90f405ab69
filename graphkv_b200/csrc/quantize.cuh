// Quantize + pack kernels (core.py:647-772, 848-910, 945-956, 979-990).
//
// Fast path: one block per tile of TT consecutive tier rows of one slice.  All
// threads gather the K and V rows of the tile into shared memory with 16-byte
// asynchronous copies, rows are rotated in place when the tensor uses the Hadamard
// rotation, then each tensor is grouped along its axis, scaled and packed straight
// to HBM.  Retained rows are copied by tiles of the same launch.
//
// General path: any geometry the tiles do not cover (group sizes that are not
// powers of two, padded head dims, tiny tiers, unaligned inputs): one thread per
// group computes the scale, one thread per output byte packs the codes.
#pragma once

#include <algorithm>

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

// Hadamard rotation of `rows` rows held in shared memory, one warp per row, by the
// 4 warps of one half-block.
template <typename T, int D>
__device__ void rotate_rows_half(T* sx, int rows, float div, float inv, int hw) {
  using G = RowGeom<T, D>;
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  for (int r = hw; r < rows; r += 4) {
    T* row = sx + r * G::kPitch + lane * EPL;
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = Elem<T>::to_f32(row[i]);
    fwht_warp<EPL>(v);
#pragma unroll
    for (int i = 0; i < EPL; ++i) row[i] = hadamard_scale<T>(v[i], div, inv);
  }
}


// Token-axis groups (keys by default): groups of gs consecutive tier rows of one
// channel.  Item = (32-bit column word w, run of 16 rows); a word holds one fp32 or
// two 16-bit channels.  Phase 1 writes every run's extrema to shared memory (red,
// [TT/16][D][2] floats); after the half-block barrier phase 2 combines the runs of
// each group, re-reads the run's values and encodes them.
template <typename T, int D, int TT, int SB, bool AFF>
__device__ void quant_token_half(const TensorDesc& d, const T* sx, int gslice, int j0, float* red, int half) {
  using G = RowGeom<T, D>;
  constexpr int W = G::kWords;
  constexpr int CPW = 4 / (int)sizeof(T);
  constexpr int RUN = kTokRun;
  constexpr int NRUN = TT / RUN;
  constexpr int ITEMS = W * NRUN;
  constexpr int ITER = (ITEMS + 127) / 128;
  constexpr int NW = (RUN * SB + 31) / 32;  // code words per channel
  constexpr int WSTRIDE = G::kPitch * (int)sizeof(T) / 4;  // row stride in 32-bit words
  const int ht = threadIdx.x & 127;
  const int rpg = d.gs / RUN;  // runs per group (host guarantees gs >= 32, a multiple of RUN)
#pragma unroll 1
  for (int itn = 0; itn < ITER; ++itn) {
    const int item = ht + itn * 128;
    if (item >= ITEMS) break;
    const int w = item % W, run = item / W;
    const uint32_t* col = reinterpret_cast<const uint32_t*>(sx + (run * RUN) * G::kPitch) + w;
    float mn[CPW], mx[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) { mn[c] = __int_as_float(0x7f800000); mx[c] = AFF ? -__int_as_float(0x7f800000) : 0.f; }
#pragma unroll
    for (int i = 0; i < RUN; ++i) {
      float f[CPW];
      unpack_word<T>(col[i * WSTRIDE], f);
#pragma unroll
      for (int c = 0; c < CPW; ++c) {
        if (AFF) { mn[c] = fminf(mn[c], f[c]); mx[c] = fmaxf(mx[c], f[c]); }
        else mx[c] = fmaxf(mx[c], fabsf(f[c]));
      }
    }
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      red[(run * D + w * CPW + c) * 2 + 0] = mn[c];
      red[(run * D + w * CPW + c) * 2 + 1] = mx[c];
    }
  }
  bar_half(half);
#pragma unroll 1
  for (int itn = 0; itn < ITER; ++itn) {
    const int item = ht + itn * 128;
    const bool act = item < ITEMS;
    const int w = act ? item % W : 0, run = act ? item / W : 0;
    const int tok0 = j0 + run * RUN;  // first tier row of the run
    const uint32_t* col = reinterpret_cast<const uint32_t*>(sx + (run * RUN) * G::kPitch) + w;
    float xf[CPW][RUN];
#pragma unroll
    for (int i = 0; i < RUN; ++i) {
      float f[CPW];
      unpack_word<T>(col[i * WSTRIDE], f);
#pragma unroll
      for (int c = 0; c < CPW; ++c) xf[c][i] = f[c];
    }
    float mn[CPW], mx[CPW];
    const int r0 = (run / rpg) * rpg;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      mn[c] = __int_as_float(0x7f800000);
      mx[c] = AFF ? -__int_as_float(0x7f800000) : 0.f;
      for (int q = 0; q < rpg; ++q) {
        if (AFF) mn[c] = fminf(mn[c], red[((r0 + q) * D + w * CPW + c) * 2 + 0]);
        mx[c] = fmaxf(mx[c], red[((r0 + q) * D + w * CPW + c) * 2 + 1]);
      }
    }
    uint32_t out[CPW][NW];
    FastCoder fc[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const GroupCoder gc = AFF ? make_affine(mn[c], mx[c], d.bits) : make_symmetric(mx[c], d.bits, d.packed != 0);
      fc[c] = fast_coder<AFF>(gc, d.packed != 0, d.bits);
      encode_run<SB, AFF, RUN>(xf[c], fc[c], out[c]);
    }
    if (act && tok0 < d.n_pad) {
#pragma unroll
      for (int c = 0; c < CPW; ++c) {
        const int ch = w * CPW + c;
        if (run % rpg == 0) {
          const int64_t gi = ((int64_t)gslice * D + ch) * d.groups_row + (tok0 >> d.log2gs);
          store_scale(d.scales, gi, d.scale_dtype, fc[c].scale);
          if (AFF) d.zps[gi] = (uint8_t)fc[c].zp;
        }
        const int64_t e0 = ((int64_t)gslice * D + ch) * d.n_pad + tok0;
        store_bytes<RUN * SB / 8>(d.codes + (e0 * SB) / 8, out[c]);
      }
    }
  }
}

// Channel-axis groups (values by default): groups of gs consecutive channels of one
// token.  Item = (tier row, run of 32 channels); the runs of a row sit in adjacent
// lanes, so group extrema combine with shuffles.
template <typename T, int D, int TT, int SB, bool AFF>
__device__ void quant_channel_half(const TensorDesc& d, const T* sx, int gslice, int j0, int rows) {
  using G = RowGeom<T, D>;
  constexpr int RPR = D / kRun;  // runs per row
  constexpr int ITEMS = TT * RPR;
  constexpr int ITER = (ITEMS + 127) / 128;
  constexpr int NW = kRun * SB / 32;
  constexpr int VPL = kRun * (int)sizeof(T) / 16;  // 16-byte vectors per run
  const int ht = threadIdx.x & 127;
  const int tpg = d.gs / kRun;  // runs (lanes) per group
#pragma unroll 1
  for (int itn = 0; itn < ITER; ++itn) {
    const int item = ht + itn * 128;
    const int r = item / RPR, run = item % RPR;
    const bool act = item < ITEMS && r < rows;
    float v[kRun];
    float mn = __int_as_float(0x7f800000), mx = AFF ? -__int_as_float(0x7f800000) : 0.f;
    if (item < ITEMS) {  // rows past the tier end hold zeros; read them to keep lanes converged
      const uint4* src = reinterpret_cast<const uint4*>(sx + r * G::kPitch + run * kRun);
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const uint4 raw = src[q];
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float f[4 / sizeof(T)];
          unpack_word<T>(wv[u], f);
#pragma unroll
          for (int e = 0; e < (int)(4 / sizeof(T)); ++e) v[(q * 4 + u) * (4 / sizeof(T)) + e] = f[e];
        }
      }
#pragma unroll
      for (int i = 0; i < kRun; ++i) {
        if (AFF) { mn = fminf(mn, v[i]); mx = fmaxf(mx, v[i]); }
        else mx = fmaxf(mx, fabsf(v[i]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < kRun; ++i) v[i] = 0.f;
    }
    for (int m = 1; m < tpg; m <<= 1) {
      if (AFF) mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, m));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, m));
    }
    const GroupCoder gc = AFF ? make_affine(mn, mx, d.bits) : make_symmetric(mx, d.bits, d.packed != 0);
    const FastCoder fc = fast_coder<AFF>(gc, d.packed != 0, d.bits);
    uint32_t out[NW];
    encode_run<SB, AFF, kRun>(v, fc, out);
    if (act) {
      const int64_t row = (int64_t)gslice * d.n + j0 + r;
      if (run % tpg == 0) {
        const int64_t gi = row * d.groups_row + run / tpg;
        store_scale(d.scales, gi, d.scale_dtype, fc.scale);
        if (AFF) d.zps[gi] = (uint8_t)fc.zp;
      }
      const int64_t e0 = row * d.n_pad + run * kRun;
      store_bytes<kRun * SB / 8>(d.codes + (e0 * SB) / 8, out);
    }
  }
}

template <typename T, int D, int TT, int SB>
__device__ __forceinline__ void quant_half_sb(const TensorDesc& d, const T* sx, int gslice, int j0, int rows,
                                              float* red, int half) {
  const bool aff = d.quantizer == GKV_AFFINE;
  if (d.axis == GKV_AXIS_TOKEN) {
    if (aff) quant_token_half<T, D, TT, SB, true>(d, sx, gslice, j0, red, half);
    else quant_token_half<T, D, TT, SB, false>(d, sx, gslice, j0, red, half);
  } else {
    if (aff) quant_channel_half<T, D, TT, SB, true>(d, sx, gslice, j0, rows);
    else quant_channel_half<T, D, TT, SB, false>(d, sx, gslice, j0, rows);
  }
}

template <typename T, int D, int TT>
__device__ __forceinline__ void quant_half(const TensorDesc& d, const T* sx, int gslice, int j0, int rows, float* red,
                                           int half) {
  if (d.sbits == 4) quant_half_sb<T, D, TT, 4>(d, sx, gslice, j0, rows, red, half);
  else if (d.sbits == 2) quant_half_sb<T, D, TT, 2>(d, sx, gslice, j0, rows, red, half);
  else quant_half_sb<T, D, TT, 8>(d, sx, gslice, j0, rows, red, half);
}

template <typename T, int D, int TT>
struct QuantTileSmem {
  using G = RowGeom<T, D>;
  static constexpr size_t kTensor = (size_t)TT * G::kPitch * sizeof(T);     // one staged tensor tile
  static constexpr size_t kBuffer = 2 * kTensor;                           // K and V
  static constexpr size_t kRed = 2 * (size_t)(TT / kTokRun) * D * 2 * sizeof(float);  // per-half run extrema
  static constexpr size_t kTotal = kBuffer + kRed;
};

template <typename T, int D, int TT>
constexpr size_t quant_tile_smem() {
  return QuantTileSmem<T, D, TT>::kTotal;
}

// Tile t of a launch -> (slice, tier, tile within the tier); tier 0 = retained rows.
struct TileRef {
  int s, tier, k;
};
__device__ __forceinline__ TileRef tile_ref(const QuantParams& p, int t) {
  TileRef r;
  r.s = t / p.tiles_slice;
  int k = t - r.s * p.tiles_slice;
  r.tier = 0;
  if (k >= p.tiles[0]) {
    k -= p.tiles[0];
    r.tier = 1;
    if (k >= p.tiles[1]) { k -= p.tiles[1]; r.tier = 2; }
  }
  r.k = k;
  return r;
}

template <typename T>
struct SliceIn {
  const T* kb;
  const T* vb;
  int64_t kst, vst;
};
template <typename T>
__device__ __forceinline__ SliceIn<T> slice_in(const QuantParams& p, int s) {
  const LayerDesc& L = p.layers[find_layer(p, s)];
  const int local = s - L.slice_begin;
  const int b = local / L.heads, h = local - b * L.heads;
  return {reinterpret_cast<const T*>(L.k) + b * L.ks[0] + h * L.ks[1],
          reinterpret_cast<const T*>(L.v) + b * L.vs[0] + h * L.vs[1], L.ks[2], L.vs[2]};
}

// Issue the 16-byte asynchronous copies that gather tile t's K and V rows into a
// staging buffer (rows past the end of the tier are zero-filled: token-axis groups
// quantize them as padding), then commit them as one group.  Retained tiles stage
// nothing but still commit a group so that the group count stays uniform.
template <typename T, int D, int TT>
__device__ __forceinline__ void stage_tile(const QuantParams& p, int t, T* sk, T* sv) {
  using G = RowGeom<T, D>;
  const TileRef tr = tile_ref(p, t);
  if (tr.tier != 0) {
    const SliceIn<T> in = slice_in<T>(p, tr.s);
    const int* idx = p.idx[tr.tier];
    const int j0 = tr.k * TT;
    const int rows = min(TT, p.n_tier[tr.tier] - j0);
    constexpr int CH = TT * G::kChunks;  // chunks per tensor
#pragma unroll
    for (int i = 0; i < 2 * CH / kThreads; ++i) {
      const int e = threadIdx.x + i * kThreads;
      const int tsr = e / CH, rem = e - tsr * CH;
      const int r = rem / G::kChunks, c = rem - r * G::kChunks;
      int tok = 0;
      if (r < rows) {
        tok = idx[j0 + r];
        if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); tok = 0; }
      }
      const T* src = (tsr ? in.vb + tok * in.vst : in.kb + tok * in.kst) + c * G::kVec;
      cp_async16((tsr ? sv : sk) + r * G::kPitch + c * G::kVec, src, r < rows ? 16u : 0u);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// One block per tile: retained-row tiles copy rows; standard / cold tiles gather
// the K and V rows into shared memory (16-byte asynchronous copies from every
// thread), then warps 0-3 quantize K and warps 4-7 quantize V, each half on its own
// named barrier.
template <typename T, int D, int TT>
__global__ void __launch_bounds__(kThreads, 3) quantize_tile_kernel(const __grid_constant__ QuantParams p,
                                                                    int total_tiles) {
  extern __shared__ __align__(128) uint8_t smem[];
  using SM = QuantTileSmem<T, D, TT>;
  (void)total_tiles;
  const int t = blockIdx.x;
  const TileRef tr = tile_ref(p, t);
  const int gslice = p.slice_offset + tr.s;
  if (tr.tier == 0) {
    const SliceIn<T> in = slice_in<T>(p, tr.s);
    copy_retained_tile<T, D>(p, in.kb, in.vb, in.kst, in.vst, gslice, tr.k);
    return;
  }
  T* sk = reinterpret_cast<T*>(smem);
  T* sv = reinterpret_cast<T*>(smem + SM::kTensor);
  float* red = reinterpret_cast<float*>(smem + SM::kBuffer);
  stage_tile<T, D, TT>(p, t, sk, sv);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  const int j0 = tr.k * TT;
  const int rows = min(TT, p.n_tier[tr.tier] - j0);
  const int half = threadIdx.x >> 7;
  const TensorDesc& d = p.t[(tr.tier == 1 ? GKV_STD_K : GKV_COLD_K) + half];
  T* sx = half ? sv : sk;
  if (d.rotation) {
    rotate_rows_half<T, D>(sx, rows, p.had_div, p.had_inv, (threadIdx.x >> 5) & 3);
    bar_half(half);
  }
  quant_half<T, D, TT>(d, sx, gslice, j0, rows, red + half * (TT / kTokRun) * D * 2, half);
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
int device_sm_count();

template <typename T, int D, int TT>
static cudaError_t launch_tile(const QuantParams& p, cudaStream_t st) {
  const size_t sm = quant_tile_smem<T, D, TT>();
  auto kern = quantize_tile_kernel<T, D, TT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  const int64_t tiles = (int64_t)p.S * p.tiles_slice;
  if (tiles == 0) return cudaSuccess;
  kern<<<(unsigned)tiles, kThreads, sm, st>>>(p, (int)tiles);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_tile_d(const QuantParams& p, cudaStream_t st) {
  if (p.D == 64) return p.tt == 64 ? launch_tile<T, 64, 64>(p, st) : launch_tile<T, 64, 128>(p, st);
  if (p.D == 128) return p.tt == 64 ? launch_tile<T, 128, 64>(p, st) : launch_tile<T, 128, 128>(p, st);
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
