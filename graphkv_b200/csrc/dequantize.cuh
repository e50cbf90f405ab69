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

#include <algorithm>

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

// ---------------------------------------------------------------------------
// Fast path: persistent blocks of 64 threads over tiles of 64 tier rows of one
// tensor, one kernel per grouping axis.  Every thread stages the packed codes of
// its items of the block's NEXT tile with asynchronous copies, and their scales,
// zero points and output rows, while it decodes the current tile -- the loads of
// a tile are in flight during the previous tile's work.  Staged codes are
// interleaved by 16-byte chunks across the block's threads (chunk q of thread t
// at (q * 64 + t) * 16), so a warp's 16-byte reads are conflict-free.
//  - channel-axis groups (V): item = (row, run of 128 bytes of output), lanes
//    mapped as in the quantizer (runs of a row 8 lanes apart); decoded, optionally
//    rotated in registers, and stored as 16-byte vectors at the output row;
//  - token-axis groups (K): item = (column word, group); decoded column-wise into
//    a shared [64][D] tile, whose rows then leave as 16-byte vectors.
// ---------------------------------------------------------------------------
constexpr int kDThreads = 64;
constexpr int kDTile = 64;
constexpr int kDItems = 4;       // items (channel axis) or item channels (token axis) per thread, at most
constexpr int kDSlot = 128;      // staged code bytes per thread and tile, at most (int8 codes)

template <typename T, int D>
struct DGeom {
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kPitchB = kRowBytes + 16;
  static constexpr int kPitchW = kPitchB / 4;
  static constexpr int kRun = 128 / (int)sizeof(T);
  static constexpr size_t kStage = (size_t)kDThreads * kDSlot;  // codes of one tile
  static constexpr size_t kMeta = (size_t)kDThreads * (2 * kDItems + 1) * 4;  // scales, zero points, output rows
  static constexpr size_t kBuf = kStage + kMeta;
  static constexpr size_t kTile = (size_t)kDTile * kPitchB;      // token-axis output tile
};

// Staging buffer of one tile: codes, then per-thread scales / zero points and
// the output row of tile row t.
struct DStage {
  uint8_t* codes;
  float* scale;  // [kDItems][64]
  int* zp;       // [kDItems][64]
  int* tok;      // [64]
  __device__ __forceinline__ static DStage at(uint8_t* base, size_t stage_bytes) {
    DStage s;
    s.codes = base;
    s.scale = reinterpret_cast<float*>(base + stage_bytes);
    s.zp = reinterpret_cast<int*>(base + stage_bytes + kDItems * kDThreads * 4);
    s.tok = reinterpret_cast<int*>(base + stage_bytes + 2 * kDItems * kDThreads * 4);
    return s;
  }
  // byte b of this thread's code slot
  __device__ __forceinline__ uint8_t* code_at(int b) const {
    return codes + ((b >> 4) * kDThreads + (int)threadIdx.x) * 16 + (b & 15);
  }
};

// Scales, zero points and the output row of a tile, loaded into registers when
// the tile's copies are issued and written to its staging buffer one tile of
// work later (so no store waits for a load).
struct DMeta {
  float scale[kDItems];
  int zp[kDItems];
  int tok;
  __device__ __forceinline__ void put(const DStage& st) const {
#pragma unroll
    for (int i = 0; i < kDItems; ++i) {
      st.scale[i * kDThreads + threadIdx.x] = scale[i];
      st.zp[i * kDThreads + threadIdx.x] = zp[i];
    }
    st.tok[threadIdx.x] = tok;
  }
};

template <int NB>
__device__ __forceinline__ void copy_codes(const DStage& st, int b0, const uint8_t* src) {
  if constexpr (NB == 8) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(st.code_at(b0))), "l"(src) : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < NB / 16; ++i) cp_async16(st.code_at(b0 + 16 * i), src + 16 * i, 16u);
  }
}

// NB (8 .. 64) staged bytes from byte b0 of this thread's slot, as words
template <int NB>
__device__ __forceinline__ void read_codes(const DStage& st, int b0, uint32_t (&w)[NB / 4]) {
  if constexpr (NB == 8) {
    const uint2 t = *reinterpret_cast<const uint2*>(st.code_at(b0));
    w[0] = t.x; w[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < NB / 16; ++i) {
      const uint4 t = *reinterpret_cast<const uint4*>(st.code_at(b0 + 16 * i));
      w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
    }
  }
}

__device__ __forceinline__ uint64_t decode_pair(uint32_t c0, uint32_t c1, uint32_t x0, uint32_t x1, uint64_t base2,
                                                uint64_t sc2) {
  return mul2(sub2(pk2(__uint_as_float(c0 ^ x0), __uint_as_float(c1 ^ x1)), base2), sc2);
}

template <typename T>
__device__ __forceinline__ uint32_t out_word(uint64_t v2) {
  return Word16<T>::round2(lo2(v2), hi2(v2));
}

struct DTileRef {
  int s, tier, k;
};
__device__ __forceinline__ DTileRef dtile_ref(const DequantParams& p, int t) {
  DTileRef r;
  r.s = (int)p.tile_div.div((uint32_t)t);
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

template <int AXIS>
__device__ __forceinline__ int dtile_role(const DequantParams& p, const DTileRef& tr, int tensor, int copy_retained) {
  if (tr.tier == 0) return copy_retained ? 1 : 0;
  return p.t[(tr.tier == 1 ? GKV_STD_K : GKV_COLD_K) + tensor].axis == AXIS ? 2 : 0;
}

// ---- channel axis ---------------------------------------------------------
template <int D, int RUN>
struct ChanMap {
  static constexpr int RPR = D / RUN;
  static constexpr int ROWS_STEP = 32 / RPR;
  static constexpr int ITEMS = (kDTile / ROWS_STEP) / 2;  // items per thread (two warps)
  __device__ __forceinline__ static void item(int i, int& r, int& u) {
    const int lane = threadIdx.x & 31, hw = threadIdx.x >> 5;
    const int j = lane & 7, k = lane >> 3;
    u = k % RPR;
    r = (hw + 2 * i) * ROWS_STEP + (k / RPR) * 8 + j;
  }
};

template <int D, int RUN, int SB>
__device__ __forceinline__ void chan_issue(const TensorDesc& d, int s, int j0, int rows, const DStage& st, DMeta& m) {
  using M = ChanMap<D, RUN>;
  constexpr int NB = RUN * SB / 8;
#pragma unroll
  for (int i = 0; i < M::ITEMS; ++i) {
    int r, u;
    M::item(i, r, u);
    float sc = 0.f;
    int zp = 0;
    if (r < rows) {
      const int64_t row = (int64_t)s * d.n + j0 + r;
      copy_codes<NB>(st, i * NB, d.codes + ((row * d.n_pad + u * RUN) * SB) / 8);
      const int64_t gi = row * d.groups_row + ((u * RUN) >> d.log2gs);
      sc = load_scale(d.scales, gi, d.scale_dtype);
      zp = load_zp(d, gi);
    }
    m.scale[i] = sc;
    m.zp[i] = zp;
  }
}

template <typename T, int D, int RUN, int SB, bool ROT>
__device__ void chan_decode(const DequantParams& p, const TensorDesc& d, const DStage& st, int rows, T* out) {
  using M = ChanMap<D, RUN>;
  constexpr int NB = RUN * SB / 8;
  constexpr int NC = NB / 4;
  constexpr int EPC = 32 / SB;
#pragma unroll 1
  for (int i = 0; i < M::ITEMS; ++i) {
    int r, u;
    M::item(i, r, u);
    const bool act = r < rows;
    uint32_t cw[NC];
    read_codes<NB>(st, i * NB, cw);
    const Decoder dc = make_decoder(d, st.scale[i * kDThreads + threadIdx.x], st.zp[i * kDThreads + threadIdx.x]);
    const uint64_t base2 = pk2(dc.base, dc.base), sc2 = pk2(dc.scale, dc.scale);
    const uint32_t xm = SB == 8 ? dc.xor_mask : 0u;  // only unpacked symmetric codes flip
    uint64_t v[RUN / 2];
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      uint32_t c[EPC];
      word_codes<SB>(cw[q], c);
#pragma unroll
      for (int e = 0; e < EPC; e += 2) v[(q * EPC + e) / 2] = decode_pair(c[e], c[e + 1], xm, xm, base2, sc2);
    }
    if constexpr (ROT) {
      // Decoded values are integer multiples of a stored scale (>= 2^-24 when
      // nonzero), so every nonzero butterfly output is far above the fused
      // quotient's 2^-100 bound.  -0 needs a zero scale (a group that underflowed
      // its scale dtype) and infinities an overflowed one: then the warp divides
      // exactly.
      const bool fused = (p.had_fused != 0) && __all_sync(kFull, dc.scale != 0.f && isfinite(dc.scale));
      rotate_run<RUN, M::RPR, false>(v, u, p.had_div, p.had_inv, fused);
    }
    const int tok = act ? st.tok[r] : -1;
    if (tok >= 0) {
      uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)tok * D + u * RUN);
      if constexpr (sizeof(T) == 4) {
#pragma unroll
        for (int k = 0; k < RUN / 2; k += 2)
          dst[k / 2] = make_uint4((uint32_t)v[k], (uint32_t)(v[k] >> 32), (uint32_t)v[k + 1], (uint32_t)(v[k + 1] >> 32));
      } else {
#pragma unroll
        for (int k = 0; k < RUN / 2; k += 4)
          dst[k / 4] = make_uint4(out_word<T>(v[k]), out_word<T>(v[k + 1]), out_word<T>(v[k + 2]), out_word<T>(v[k + 3]));
      }
    }
  }
}

// ---- token axis -----------------------------------------------------------
template <typename T, int D, int GS>
struct TokMap {
  static constexpr int W = D * (int)sizeof(T) / 4;       // column words
  static constexpr int CPW = 4 / (int)sizeof(T);         // channels per word
  static constexpr int ITEMS_TILE = W * (kDTile / GS);
  static constexpr int ITEMS = (ITEMS_TILE + kDThreads - 1) / kDThreads;
};

template <typename T, int D, int GS, int SB>
__device__ __forceinline__ void tok_issue(const TensorDesc& d, int s, int j0, const DStage& st, DMeta& m) {
  using M = TokMap<T, D, GS>;
  constexpr int NB = GS * SB / 8;  // code bytes per channel and group
#pragma unroll
  for (int i = 0; i < M::ITEMS; ++i) {
    const int item = threadIdx.x + i * kDThreads;
    const int g = item / M::W, w = item - g * M::W;
    const int tok0 = j0 + g * GS;
#pragma unroll
    for (int c = 0; c < M::CPW; ++c) {
      float sc = 0.f;
      int zp = 0;
      if (item < M::ITEMS_TILE && tok0 < d.n_pad) {
        const int64_t crow = (int64_t)s * D + w * M::CPW + c;
        copy_codes<NB>(st, (i * M::CPW + c) * NB, d.codes + ((crow * d.n_pad + tok0) * SB) / 8);
        const int64_t gi = crow * d.groups_row + (tok0 >> d.log2gs);
        sc = load_scale(d.scales, gi, d.scale_dtype);
        zp = load_zp(d, gi);
      }
      m.scale[i * M::CPW + c] = sc;
      m.zp[i * M::CPW + c] = zp;
    }
  }
}

template <typename T, int D, int GS, int SB>
__device__ void tok_decode(const TensorDesc& d, const DStage& st, int j0, uint8_t* tile) {
  using M = TokMap<T, D, GS>;
  using G = DGeom<T, D>;
  constexpr int NB = GS * SB / 8;
  constexpr int NC = NB / 4;
  constexpr int EPC = 32 / SB;
#pragma unroll 1
  for (int i = 0; i < M::ITEMS; ++i) {
    const int item = threadIdx.x + i * kDThreads;
    if (item >= M::ITEMS_TILE) break;
    const int g = item / M::W, w = item - g * M::W;
    if (j0 + g * GS >= d.n_pad) continue;
    uint32_t* col = reinterpret_cast<uint32_t*>(tile + (g * GS) * G::kPitchB) + w;
    if constexpr (M::CPW == 2) {
      const int k0 = (2 * i) * kDThreads + threadIdx.x, k1 = k0 + kDThreads;
      const Decoder d0 = make_decoder(d, st.scale[k0], st.zp[k0]);
      const Decoder d1 = make_decoder(d, st.scale[k1], st.zp[k1]);
      const uint64_t base2 = pk2(d0.base, d1.base), sc2 = pk2(d0.scale, d1.scale);
      const uint32_t x0 = SB == 8 ? d0.xor_mask : 0u, x1 = SB == 8 ? d1.xor_mask : 0u;
      uint32_t c0w[NC], c1w[NC];
      read_codes<NB>(st, (2 * i) * NB, c0w);
      read_codes<NB>(st, (2 * i + 1) * NB, c1w);
#pragma unroll
      for (int q = 0; q < NC; ++q) {
        uint32_t a[EPC], b[EPC];
        word_codes<SB>(c0w[q], a);
        word_codes<SB>(c1w[q], b);
#pragma unroll
        for (int e = 0; e < EPC; ++e)
          col[(q * EPC + e) * G::kPitchW] = out_word<T>(decode_pair(a[e], b[e], x0, x1, base2, sc2));
      }
    } else {
      const int k0 = i * kDThreads + threadIdx.x;
      const Decoder d0 = make_decoder(d, st.scale[k0], st.zp[k0]);
      const uint64_t base2 = pk2(d0.base, d0.base), sc2 = pk2(d0.scale, d0.scale);
      const uint32_t x0 = SB == 8 ? d0.xor_mask : 0u;
      uint32_t cw[NC];
      read_codes<NB>(st, i * NB, cw);
#pragma unroll
      for (int q = 0; q < NC; ++q) {
        uint32_t a[EPC];
        word_codes<SB>(cw[q], a);
#pragma unroll
        for (int e = 0; e < EPC; e += 2) {
          const uint64_t v2 = decode_pair(a[e], a[e + 1], x0, x0, base2, sc2);
          col[(q * EPC + e) * G::kPitchW] = (uint32_t)v2;
          col[(q * EPC + e + 1) * G::kPitchW] = (uint32_t)(v2 >> 32);
        }
      }
    }
  }
}

// ---- dispatch -------------------------------------------------------------
template <typename T, int D, int AXIS>
__device__ __forceinline__ void dq_issue(const TensorDesc& d, int s, int j0, int rows, const DStage& st, DMeta& m) {
  if constexpr (AXIS == GKV_AXIS_TOKEN) {
    (void)rows;
    if (d.gs == 64) {
      if (d.sbits == 4) tok_issue<T, D, 64, 4>(d, s, j0, st, m);
      else if (d.sbits == 2) tok_issue<T, D, 64, 2>(d, s, j0, st, m);
      else tok_issue<T, D, 64, 8>(d, s, j0, st, m);
    } else {
      if (d.sbits == 4) tok_issue<T, D, 32, 4>(d, s, j0, st, m);
      else if (d.sbits == 2) tok_issue<T, D, 32, 2>(d, s, j0, st, m);
      else tok_issue<T, D, 32, 8>(d, s, j0, st, m);
    }
  } else {
    constexpr int RUN = DGeom<T, D>::kRun;
    if (d.gs < RUN) {
      if constexpr (RUN / 2 >= 32 && D / (RUN / 2) <= 4) {
        if (d.sbits == 4) chan_issue<D, RUN / 2, 4>(d, s, j0, rows, st, m);
        else if (d.sbits == 2) chan_issue<D, RUN / 2, 2>(d, s, j0, rows, st, m);
        else chan_issue<D, RUN / 2, 8>(d, s, j0, rows, st, m);
      }
    } else {
      if (d.sbits == 4) chan_issue<D, RUN, 4>(d, s, j0, rows, st, m);
      else if (d.sbits == 2) chan_issue<D, RUN, 2>(d, s, j0, rows, st, m);
      else chan_issue<D, RUN, 8>(d, s, j0, rows, st, m);
    }
  }
}

template <typename T, int D, int RUN>
__device__ __forceinline__ void chan_decode_any(const DequantParams& p, const TensorDesc& d, const DStage& st, int rows,
                                                T* out) {
  if (d.rotation) {
    if (d.sbits == 4) chan_decode<T, D, RUN, 4, true>(p, d, st, rows, out);
    else if (d.sbits == 2) chan_decode<T, D, RUN, 2, true>(p, d, st, rows, out);
    else chan_decode<T, D, RUN, 8, true>(p, d, st, rows, out);
  } else {
    if (d.sbits == 4) chan_decode<T, D, RUN, 4, false>(p, d, st, rows, out);
    else if (d.sbits == 2) chan_decode<T, D, RUN, 2, false>(p, d, st, rows, out);
    else chan_decode<T, D, RUN, 8, false>(p, d, st, rows, out);
  }
}

// Persistent blocks over the tiles of one tensor (`tensor` 1: values, 0: keys),
// compiled per grouping axis; retained-row tiles are copied when `copy_retained`.
template <typename T, int D, int AXIS>
__global__ void __launch_bounds__(kDThreads, AXIS == GKV_AXIS_TOKEN ? 5 : 8) dequantize_tile_kernel(const __grid_constant__ DequantParams p,
                                                                       int tensor, int copy_retained,
                                                                       int total_tiles) {
  extern __shared__ __align__(128) uint8_t smem[];
  using G = DGeom<T, D>;
  uint8_t* tile = smem + 2 * G::kBuf;  // token axis: [64][pitch]
  T* const out_base = reinterpret_cast<T*>(tensor ? p.out_v : p.out_k);
  int cur = blockIdx.x, role = 0;
  for (; cur < total_tiles; cur += gridDim.x)
    if ((role = dtile_role<AXIS>(p, dtile_ref(p, cur), tensor, copy_retained)) != 0) break;
  int buf = 0;
  // issue the copies of tile t into buffer b; its metadata comes back in registers
  auto issue = [&](int t, int b) {
    DMeta m;
#pragma unroll
    for (int i = 0; i < kDItems; ++i) { m.scale[i] = 0.f; m.zp[i] = 0; }
    const DTileRef tr = dtile_ref(p, t);
    const TensorDesc& d = p.t[(tr.tier == 1 ? GKV_STD_K : GKV_COLD_K) + tensor];
    const int j0 = tr.k * kDTile;
    const int rows = min(kDTile, p.n_tier[tr.tier] - j0);
    dq_issue<T, D, AXIS>(d, tr.s, j0, rows, DStage::at(smem + b * G::kBuf, G::kStage), m);
    m.tok = -1;
    if ((int)threadIdx.x < rows) {
      m.tok = p.idx[tr.tier][j0 + threadIdx.x];
      if ((unsigned)m.tok >= (unsigned)p.T) { raise_error(kErrBadIndex); m.tok = -1; }
    }
    return m;
  };
  if (cur < total_tiles && role == 2) issue(cur, 0).put(DStage::at(smem, G::kStage));
  asm volatile("cp.async.commit_group;" ::: "memory");
  while (cur < total_tiles) {
    int nxt = cur + gridDim.x, nrole = 0;
    for (; nxt < total_tiles; nxt += gridDim.x)
      if ((nrole = dtile_role<AXIS>(p, dtile_ref(p, nxt), tensor, copy_retained)) != 0) break;
    const bool stage_next = nxt < total_tiles && nrole == 2;
    DMeta next_meta;
    if (stage_next) next_meta = issue(nxt, buf ^ 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const DTileRef tr = dtile_ref(p, cur);
    T* out = out_base + (int64_t)tr.s * p.T * D;
    if (role == 1) {
      // retained rows: thread = (16-byte chunk, rows r0, r0 + STEP, ...), loads before stores
      constexpr int VEC = 16 / (int)sizeof(T), CPR = D / VEC, STEP = kDThreads / CPR, N = kRetTile / STEP;
      const int R = p.n_tier[0];
      const int j0 = tr.k * kRetTile, rows = min(kRetTile, R - j0);
      const T* src = reinterpret_cast<const T*>(tensor ? p.ret_v : p.ret_k) + ((int64_t)tr.s * R + j0) * D;
      const int c = threadIdx.x % CPR, r0 = threadIdx.x / CPR;
      uint4 v[N];
      int to[N];
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int r = r0 + i * STEP;
        to[i] = -1;
        v[i] = make_uint4(0u, 0u, 0u, 0u);
        if (r < rows) {
          to[i] = p.idx[0][j0 + r];
          if ((unsigned)to[i] >= (unsigned)p.T) { raise_error(kErrBadIndex); to[i] = -1; }
          v[i] = *reinterpret_cast<const uint4*>(src + r * D + c * VEC);
        }
      }
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (to[i] >= 0) *reinterpret_cast<uint4*>(out + (int64_t)to[i] * D + c * VEC) = v[i];
    } else {
      asm volatile("cp.async.wait_group 1;" ::: "memory");
      __syncthreads();  // every thread's staged rows / metadata of this tile are visible
      const TensorDesc& d = p.t[(tr.tier == 1 ? GKV_STD_K : GKV_COLD_K) + tensor];
      const int j0 = tr.k * kDTile;
      const int rows = min(kDTile, p.n_tier[tr.tier] - j0);
      const DStage st = DStage::at(smem + buf * G::kBuf, G::kStage);
      if constexpr (AXIS == GKV_AXIS_TOKEN) {
        if (d.gs == 64) {
          if (d.sbits == 4) tok_decode<T, D, 64, 4>(d, st, j0, tile);
          else if (d.sbits == 2) tok_decode<T, D, 64, 2>(d, st, j0, tile);
          else tok_decode<T, D, 64, 8>(d, st, j0, tile);
        } else {
          if (d.sbits == 4) tok_decode<T, D, 32, 4>(d, st, j0, tile);
          else if (d.sbits == 2) tok_decode<T, D, 32, 2>(d, st, j0, tile);
          else tok_decode<T, D, 32, 8>(d, st, j0, tile);
        }
        // the tile's rows leave as 16-byte vectors: thread = (chunk, rows r0, r0 + step, ...)
        __syncthreads();
        constexpr int CH = G::kRowBytes / 16, STEP = kDThreads / CH;
        const int c = threadIdx.x % CH, r0 = threadIdx.x / CH;
#pragma unroll 4
        for (int i = 0; i < kDTile / STEP; ++i) {
          const int r = r0 + i * STEP;
          const int t_out = r < rows ? st.tok[r] : -1;
          if (t_out >= 0)
            reinterpret_cast<uint4*>(out + (int64_t)t_out * D)[c] =
                *reinterpret_cast<const uint4*>(tile + r * G::kPitchB + c * 16);
        }
      } else {
        constexpr int RUN = G::kRun;
        if (d.gs < RUN) {
          if constexpr (RUN / 2 >= 32 && D / (RUN / 2) <= 4) chan_decode_any<T, D, RUN / 2>(p, d, st, rows, out);
        } else {
          chan_decode_any<T, D, RUN>(p, d, st, rows, out);
        }
      }
    }
    if (stage_next) next_meta.put(DStage::at(smem + (buf ^ 1) * G::kBuf, G::kStage));
    __syncthreads();  // this buffer and the tile are rewritten from the next iteration on
    cur = nxt;
    role = nrole;
    buf ^= 1;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
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
template <typename T, int D>
static cudaError_t launch_dq_tile(const DequantParams& p, cudaStream_t st) {
  using G = DGeom<T, D>;
  const int64_t tiles = (int64_t)p.S * p.tiles_slice;
  if (tiles == 0) return cudaSuccess;
  const size_t sm_ch = 2 * G::kBuf;
  const size_t sm_tok = sm_ch + G::kTile;
  auto ktok = dequantize_tile_kernel<T, D, GKV_AXIS_TOKEN>;
  auto kch = dequantize_tile_kernel<T, D, GKV_AXIS_CHANNEL>;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(ktok, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_tok)) != cudaSuccess)
    return e;
  if ((e = cudaFuncSetAttribute(kch, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_ch)) != cudaSuccess)
    return e;
  int occ_tok = 0, occ_ch = 0;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_tok, ktok, kDThreads, sm_tok)) != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_ch, kch, kDThreads, sm_ch)) != cudaSuccess) return e;
  const int sms = device_sm_count();
  const unsigned g_tok = (unsigned)std::min<int64_t>(tiles, (int64_t)sms * std::max(occ_tok, 1));
  const unsigned g_ch = (unsigned)std::min<int64_t>(tiles, (int64_t)sms * std::max(occ_ch, 1));
  for (int tensor = 0; tensor < 2; ++tensor) {
    bool token = false, channel = false;
    for (int tier = 1; tier <= 2; ++tier) {
      if (p.tiles[tier] == 0) continue;
      const TensorDesc& d = p.t[(tier == 1 ? GKV_STD_K : GKV_COLD_K) + tensor];
      (d.axis == GKV_AXIS_TOKEN ? token : channel) = true;
    }
    if (!token && !channel) channel = true;  // retained rows only
    if (token) ktok<<<g_tok, kDThreads, sm_tok, st>>>(p, tensor, 1, (int)tiles);
    if (channel) kch<<<g_ch, kDThreads, sm_ch, st>>>(p, tensor, token ? 0 : 1, (int)tiles);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

template <typename T>
static cudaError_t launch_dq_tile_d(const DequantParams& p, cudaStream_t st) {
  if (p.D == 64) return launch_dq_tile<T, 64>(p, st);
  if (p.D == 128) return launch_dq_tile<T, 128>(p, st);
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
