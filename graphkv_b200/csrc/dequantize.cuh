// Unpack + dequantize + scatter kernels (core.py:153-173, 265-307, 993-1007).
//
// Every output row [s, t, :] is written exactly once: retained rows are copied
// from the retained store, standard and cold rows are decoded from their tiers.
// Decoded values are (q - zp) * scale in fp32 (one rounding, no FMA), then the
// optional inverse Hadamard (the same butterflies, fp32), then the cast to the
// cache dtype.
//
// Fast path: one block of 128 threads per tile of 64 tier rows of one slice and
// tensor.  Token-axis tensors decode column runs (thread per 32-bit column word
// and run of 32 rows), channel-axis tensors decode row runs (thread per 128-byte
// run, rotated runs through in-register butterflies); both decode into a shared
// [64][D] tile whose rows leave as whole 256-byte rows of 16-byte stores.
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
// Fast path: one block of 128 threads per tile of 64 tier rows of one tensor,
// one kernel per grouping axis; many blocks per SM, each thread loading its
// codes, scales and output rows straight into registers (the other resident
// warps cover the latency).
//  - channel-axis groups (V): item = (row, run of 128 bytes of output), lanes
//    mapped as in the quantizer (runs of a row 8 lanes apart); decoded and
//    optionally rotated in registers;
//  - token-axis groups (K): item = (column word, run of 32 rows); decoded
//    column-wise;
// both into a shared [64][D] tile whose rows then leave as 16-byte vectors, 16
// lanes per row (whole 32-byte sectors per store instruction).
// ---------------------------------------------------------------------------
constexpr int kDThreads = 128;
constexpr int kDWarps = kDThreads / 32;
constexpr int kDTile = 64;
constexpr int kDRows = 32;  // rows of a token-axis column run

template <typename T, int D>
struct DGeom {
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kPitchB = kRowBytes + 16;
  static constexpr int kPitchW = kPitchB / 4;
  static constexpr int kWords = kRowBytes / 4;
  static constexpr int kRun = 128 / (int)sizeof(T);
  static constexpr size_t kTile = (size_t)kDTile * kPitchB;  // token-axis output tile
};

template <int NB>
__device__ __forceinline__ void load_codes(const uint8_t* src, uint32_t (&w)[NB / 4]) {
  if constexpr (NB == 8) {
    const uint2 t = *reinterpret_cast<const uint2*>(src);
    w[0] = t.x; w[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < NB / 16; ++i) {
      const uint4 t = reinterpret_cast<const uint4*>(src)[i];
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

// output rows of a tile in shared memory (-1: none)
__device__ __forceinline__ void load_tile_rows(const DequantParams& p, const DTileRef& tr, int j0, int rows, int* toks) {
  for (int r = threadIdx.x; r < kDTile; r += kDThreads) {
    int t = -1;
    if (r < rows) {
      t = p.idx[tr.tier][j0 + r];
      if ((unsigned)t >= (unsigned)p.T) { raise_error(kErrBadIndex); t = -1; }
    }
    toks[r] = t;
  }
}

// ---- channel axis ---------------------------------------------------------
template <typename T, int D, int RUN, int SB, bool ROT>
__device__ void chan_decode(const DequantParams& p, const TensorDesc& d, int s, int j0, int rows, uint8_t* tile) {
  constexpr int RPR = D / RUN;
  constexpr int ROWS_STEP = 32 / RPR;
  constexpr int STEPS = kDTile / ROWS_STEP;
  constexpr int NB = RUN * SB / 8;
  constexpr int NC = NB / 4;
  constexpr int EPC = 32 / SB;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = lane & 7, k = lane >> 3;
  const int u = k % RPR, rb = k / RPR;
#pragma unroll 1
  for (int step = warp; step < STEPS; step += kDWarps) {
    const int r = step * ROWS_STEP + rb * 8 + j;
    const bool act = r < rows;
    uint32_t cw[NC];
    float scale = 0.f;
    int zp = 0;
    if (act) {
      const int64_t row = (int64_t)s * d.n + j0 + r;
      load_codes<NB>(d.codes + ((row * d.n_pad + u * RUN) * SB) / 8, cw);
      const int64_t gi = row * d.groups_row + ((u * RUN) >> d.log2gs);
      scale = load_scale(d.scales, gi, d.scale_dtype);
      zp = load_zp(d, gi);
    } else {
#pragma unroll
      for (int q = 0; q < NC; ++q) cw[q] = 0u;
    }
    const Decoder dc = make_decoder(d, scale, zp);
    const uint64_t base2 = pk2(dc.base, dc.base), sc2 = pk2(dc.scale, dc.scale);
    const uint32_t xm = SB == 8 ? dc.xor_mask : 0u;  // only unpacked symmetric codes flip
    uint4* dst = reinterpret_cast<uint4*>(tile + r * DGeom<T, D>::kPitchB + u * RUN * (int)sizeof(T));
    if constexpr (!ROT) {
      // decode and write 16 bytes of output at a time (few live registers)
      constexpr int OC = 16 / (int)sizeof(T);  // output elements per 16-byte store
#pragma unroll
      for (int o = 0; o < RUN / OC; ++o) {
        uint32_t c[OC];
#pragma unroll
        for (int q = 0; q < (OC + EPC - 1) / EPC; ++q) {  // the code words covering this chunk
          const int e0 = o * OC + q * EPC;
          uint32_t all[EPC];
          word_codes<SB>(cw[e0 / EPC], all);
#pragma unroll
          for (int e = 0; e < (EPC < OC ? EPC : OC); ++e) c[q * EPC + e] = all[(e0 % EPC) + e];
        }
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < OC; e += 2) {
          const uint64_t v2 = decode_pair(c[e], c[e + 1], xm, xm, base2, sc2);
          if constexpr (sizeof(T) == 4) { w[e] = lo32(v2); w[e + 1] = hi32(v2); }
          else w[e / 2] = out_word<T>(v2);
        }
        dst[o] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
      uint64_t v[RUN / 2];
#pragma unroll
      for (int q = 0; q < NC; ++q) {
        uint32_t c[EPC];
        word_codes<SB>(cw[q], c);
#pragma unroll
        for (int e = 0; e < EPC; e += 2) v[(q * EPC + e) / 2] = decode_pair(c[e], c[e + 1], xm, xm, base2, sc2);
      }
      // Decoded values are integer multiples of a stored scale (>= 2^-24 when
      // nonzero), so every nonzero butterfly output is far above the fused
      // quotient's 2^-100 bound.  -0 needs a zero scale (a group that underflowed
      // its scale dtype) and infinities an overflowed one: then the warp divides
      // exactly.  (Padding lanes hold scale 0 but only zeros: they do not vote.)
      const bool fused = (p.had_fused != 0) && __all_sync(kFull, !act || (dc.scale != 0.f && isfinite(dc.scale)));
      rotate_run<RUN, RPR, false>(v, u, p.had_div, p.had_inv, fused);
      if constexpr (sizeof(T) == 4) {
#pragma unroll
        for (int q = 0; q < RUN / 2; q += 2)
          dst[q / 2] = make_uint4(lo32(v[q]), hi32(v[q]), lo32(v[q + 1]), hi32(v[q + 1]));
      } else {
#pragma unroll
        for (int q = 0; q < RUN / 2; q += 4)
          dst[q / 4] = make_uint4(out_word<T>(v[q]), out_word<T>(v[q + 1]), out_word<T>(v[q + 2]), out_word<T>(v[q + 3]));
      }
    }
  }
}

// ---- token axis -----------------------------------------------------------
template <typename T, int D, int SB>
__device__ void tok_decode(const TensorDesc& d, int s, int j0, uint8_t* tile) {
  using G = DGeom<T, D>;
  constexpr int CPW = 4 / (int)sizeof(T);
  constexpr int NH = kDTile / kDRows;
  constexpr int ITEMS = G::kWords * NH;
  constexpr int NB = kDRows * SB / 8;  // code bytes per channel and run
  constexpr int NC = NB / 4;
  constexpr int EPC = 32 / SB;
#pragma unroll 1
  for (int item = threadIdx.x; item < ITEMS; item += kDThreads) {
    const int h = item / G::kWords, w = item - h * G::kWords;
    const int tok0 = j0 + h * kDRows;
    if (tok0 >= d.n_pad) continue;
    uint32_t* col = reinterpret_cast<uint32_t*>(tile + (h * kDRows) * G::kPitchB) + w;
    if constexpr (CPW == 2) {
      const int64_t crow = (int64_t)s * D + 2 * w;
      uint32_t c0w[NC], c1w[NC];
      load_codes<NB>(d.codes + ((crow * d.n_pad + tok0) * SB) / 8, c0w);
      load_codes<NB>(d.codes + (((crow + 1) * d.n_pad + tok0) * SB) / 8, c1w);
      const int64_t gi = crow * d.groups_row + (tok0 >> d.log2gs);
      const Decoder d0 = make_decoder(d, load_scale(d.scales, gi, d.scale_dtype), load_zp(d, gi));
      const Decoder d1 = make_decoder(d, load_scale(d.scales, gi + d.groups_row, d.scale_dtype),
                                      load_zp(d, gi + d.groups_row));
      const uint64_t base2 = pk2(d0.base, d1.base), sc2 = pk2(d0.scale, d1.scale);
      const uint32_t x0 = SB == 8 ? d0.xor_mask : 0u, x1 = SB == 8 ? d1.xor_mask : 0u;
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
      const int64_t crow = (int64_t)s * D + w;
      uint32_t cw[NC];
      load_codes<NB>(d.codes + ((crow * d.n_pad + tok0) * SB) / 8, cw);
      const int64_t gi = crow * d.groups_row + (tok0 >> d.log2gs);
      const Decoder d0 = make_decoder(d, load_scale(d.scales, gi, d.scale_dtype), load_zp(d, gi));
      const uint64_t base2 = pk2(d0.base, d0.base), sc2 = pk2(d0.scale, d0.scale);
      const uint32_t x0 = SB == 8 ? d0.xor_mask : 0u;
#pragma unroll
      for (int q = 0; q < NC; ++q) {
        uint32_t a[EPC];
        word_codes<SB>(cw[q], a);
#pragma unroll
        for (int e = 0; e < EPC; e += 2) {
          const uint64_t v2 = decode_pair(a[e], a[e + 1], x0, x0, base2, sc2);
          col[(q * EPC + e) * G::kPitchW] = lo32(v2);
          col[(q * EPC + e + 1) * G::kPitchW] = hi32(v2);
        }
      }
    }
  }
}

// ---- rotated channel axis, 16-bit rows of 128 -----------------------------
// Two threads per row, thread u (lane bit 3) decoding elements 64u .. 64u + 63
// (one group of 64, or half of a group of 128) as 32 packed fp32 pairs.  The
// decoded values are integer codes times one stored scale per group, so the
// butterfly stages h = 1 .. 32, which stay inside a group, are exact in fp32
// (at most 64 codes of magnitude <= 128 per sum, times a 16-bit-mantissa
// scale); only h = 64 mixes the two groups' scales and rounds, as in the
// reference.  As in the quantizer, thread 1 holds its halves swapped so that
// both threads hand over pairs 16 .. 31, and the h = 64 stage pairs element e of
// the two halves through the threads' own 128 bytes of the output tile row.
// Unlike codes, output bits carry the sign of zero, so the h = 64 sums and
// differences are formed with the reference's operand order (below).
template <typename T, int SB>
__device__ void dequant_rot_pair(const DequantParams& p, const TensorDesc& d, int s, int j0, int rows,
                                 uint8_t* tile) {
  using G = DGeom<T, 128>;
  using W = Word16<T>;
  constexpr int HB = 4 * SB;   // code bytes of 32 elements
  constexpr int HC = HB / 4;   // code words of 32 elements
  constexpr int EPC = 32 / SB;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = lane & 7, k = lane >> 3;
  const int u = k & 1, rb = k >> 1;
  const float sg = u ? -1.f : 1.f;
  const uint64_t sgp = pk2(sg, sg), sgn = pk2(-sg, -sg);
#pragma unroll 1
  for (int step = warp; step < kDTile / 16; step += kDWarps) {
    const int r = step * 16 + rb * 8 + j;
    const bool act = r < rows;
    uint32_t h0[HC], h1[HC];
    float scale = 0.f;
    int zp = 0;
    if (act) {
      const int64_t row = (int64_t)s * d.n + j0 + r;
      const uint8_t* src = d.codes + ((row * d.n_pad + 64 * u) * SB) / 8;
      load_codes<HB>(src + (u ? HB : 0), h0);
      load_codes<HB>(src + (u ? 0 : HB), h1);
      const int64_t gi = row * d.groups_row + ((64 * u) >> d.log2gs);
      scale = load_scale(d.scales, gi, d.scale_dtype);
      zp = load_zp(d, gi);
    } else {
#pragma unroll
      for (int q = 0; q < HC; ++q) h0[q] = h1[q] = 0u;
    }
    const Decoder dc = make_decoder(d, scale, zp);
    const uint64_t base2 = pk2(dc.base, dc.base), sc2 = pk2(dc.scale, dc.scale);
    const uint32_t xm = SB == 8 ? dc.xor_mask : 0u;
    uint64_t v[32];
#pragma unroll
    for (int q = 0; q < HC; ++q) {
      uint32_t c0[EPC], c1[EPC];
      word_codes<SB>(h0[q], c0);
      word_codes<SB>(h1[q], c1);
#pragma unroll
      for (int e = 0; e < EPC; e += 2) {
        v[(q * EPC + e) / 2] = decode_pair(c0[e], c0[e + 1], xm, xm, base2, sc2);
        v[16 + (q * EPC + e) / 2] = decode_pair(c1[e], c1[e + 1], xm, xm, base2, sc2);
      }
    }
    // h = 1 (inside each pair), h = 2 .. 16, h = 32 (thread 1: lower element in m + 16)
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      const float a = lo2(v[m]), b = hi2(v[m]);
      v[m] = pk2(__fadd_rn(a, b), __fsub_rn(a, b));
    }
#pragma unroll
    for (int h = 2; h < 32; h <<= 1) {
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        if ((2 * m) & h) continue;
        const uint64_t a = v[m], b = v[m + h / 2];
        v[m] = add2(a, b);
        v[m + h / 2] = sub2(a, b);
      }
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const uint64_t a = v[m], b = v[m + 16];
      v[m] = fma2(sgp, a, b);
      v[m + 16] = fma2(sgn, b, a);
    }
    // Nonzero decoded values are >= 2^-24 (a code times a stored scale), so the
    // fused quotient is exact; -0 needs a zero scale and infinities an overflowed
    // one, and then the warp divides exactly (padding rows hold zeros only).
    const bool fused = (p.had_fused != 0) && __all_sync(kFull, !act || (scale != 0.f && isfinite(scale)));
    uint8_t* own = tile + r * G::kPitchB + u * 128;
    uint4* mine = reinterpret_cast<uint4*>(own);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      mine[q] = make_uint4(lo32(v[16 + 2 * q]), hi32(v[16 + 2 * q]), lo32(v[17 + 2 * q]), hi32(v[17 + 2 * q]));
    __syncwarp();
    const uint4* theirs = reinterpret_cast<const uint4*>(tile + r * G::kPitchB + (u ^ 1) * 128);
    uint32_t ws[16], wd[16];
    const uint64_t nd2 = pk2(-p.had_div, -p.had_div), rd2 = pk2(p.had_inv, p.had_inv);
    // Sums a + b and differences a - b of the two halves' elements with the
    // reference's zero signs (a: thread 0's values, b: thread 1's): thread 0
    // negates what it receives (-b) and forms a + (-b) and (-1)(-b) + a, thread 1
    // forms (-1) b + a and a + b -- in IEEE arithmetic x - y is x + (-y), and the
    // products with -1 are exact.
    const uint32_t nm = u ? 0u : 0x80000000u;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 t = theirs[q];
      const uint64_t o0 = pk2u(t.x ^ nm, t.y ^ nm), o1 = pk2u(t.z ^ nm, t.w ^ nm);
      uint64_t s0 = fma2(sgn, o0, v[2 * q]), s1 = fma2(sgn, o1, v[2 * q + 1]);
      uint64_t d0 = fma2(sgp, v[2 * q], o0), d1 = fma2(sgp, v[2 * q + 1], o1);
      if (fused) {
        s0 = quot2(s0, nd2, rd2);
        s1 = quot2(s1, nd2, rd2);
        d0 = quot2(d0, nd2, rd2);
        d1 = quot2(d1, nd2, rd2);
      } else {
        const float dv = p.had_div;
        s0 = pk2(__fdiv_rn(lo2(s0), dv), __fdiv_rn(hi2(s0), dv));
        s1 = pk2(__fdiv_rn(lo2(s1), dv), __fdiv_rn(hi2(s1), dv));
        d0 = pk2(__fdiv_rn(lo2(d0), dv), __fdiv_rn(hi2(d0), dv));
        d1 = pk2(__fdiv_rn(lo2(d1), dv), __fdiv_rn(hi2(d1), dv));
      }
      ws[2 * q] = W::round2(lo2(s0), hi2(s0));
      ws[2 * q + 1] = W::round2(lo2(s1), hi2(s1));
      wd[2 * q] = W::round2(lo2(d0), hi2(d0));
      wd[2 * q + 1] = W::round2(lo2(d1), hi2(d1));
    }
    __syncwarp();  // the partner has read this thread's half row
    uint4* out_s = reinterpret_cast<uint4*>(tile + r * G::kPitchB + 64 * u);
    uint4* out_d = reinterpret_cast<uint4*>(tile + r * G::kPitchB + 128 + 64 * u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      out_s[i] = make_uint4(ws[4 * i], ws[4 * i + 1], ws[4 * i + 2], ws[4 * i + 3]);
      out_d[i] = make_uint4(wd[4 * i], wd[4 * i + 1], wd[4 * i + 2], wd[4 * i + 3]);
    }
  }
}

template <typename T, int D, int RUN, bool ROT>
__device__ __forceinline__ void chan_decode_any(const DequantParams& p, const TensorDesc& d, int s, int j0, int rows,
                                                uint8_t* tile) {
  if constexpr (ROT && D == 128 && sizeof(T) == 2) {
    if (d.gs >= 64) {
      if (d.sbits == 4) dequant_rot_pair<T, 4>(p, d, s, j0, rows, tile);
      else if (d.sbits == 2) dequant_rot_pair<T, 2>(p, d, s, j0, rows, tile);
      else dequant_rot_pair<T, 8>(p, d, s, j0, rows, tile);
      return;
    }
  }
  if (d.sbits == 4) chan_decode<T, D, RUN, 4, ROT>(p, d, s, j0, rows, tile);
  else if (d.sbits == 2) chan_decode<T, D, RUN, 2, ROT>(p, d, s, j0, rows, tile);
  else chan_decode<T, D, RUN, 8, ROT>(p, d, s, j0, rows, tile);
}

// One block per tile of one tensor (`tensor` 1: values, 0: keys).  Compiled per
// grouping axis and rotation (channel axis only: rotated token-axis tensors take
// the general path); a launch covers the tiers that use its variant, and the
// retained rows when `copy_retained`.
template <typename T, int D, int AXIS, bool ROT>
__global__ void __launch_bounds__(kDThreads, sizeof(T) == 4 ? (AXIS == GKV_AXIS_TOKEN ? 7 : (ROT ? 5 : 10)) : (AXIS == GKV_AXIS_TOKEN ? 8 : (ROT ? 7 : 10)))
    dequantize_tile_kernel(const __grid_constant__ DequantParams p, int tensor, int copy_retained) {
  extern __shared__ __align__(128) uint8_t smem[];
  using G = DGeom<T, D>;
  const DTileRef tr = dtile_ref(p, blockIdx.x);
  if (tr.tier == 0 && !copy_retained) return;
  const TensorDesc& d = p.t[(tr.tier == 1 ? GKV_STD_K : GKV_COLD_K) + tensor];
  if (tr.tier != 0 && (d.axis != AXIS || (d.rotation != 0) != ROT)) return;
  T* out = reinterpret_cast<T*>(tensor ? p.out_v : p.out_k) + (int64_t)tr.s * p.out_T * D;
  if (tr.tier == 0) {
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
    return;
  }
  const int j0 = tr.k * kDTile;
  const int rows = min(kDTile, p.n_tier[tr.tier] - j0);
  uint8_t* tile = smem;
  int* toks = reinterpret_cast<int*>(smem + G::kTile);
  load_tile_rows(p, tr, j0, rows, toks);
  if constexpr (AXIS == GKV_AXIS_TOKEN) {
    if (d.sbits == 4) tok_decode<T, D, 4>(d, tr.s, j0, tile);
    else if (d.sbits == 2) tok_decode<T, D, 2>(d, tr.s, j0, tile);
    else tok_decode<T, D, 8>(d, tr.s, j0, tile);
  } else {
    constexpr int RUN = G::kRun;
    // rotated runs are half as long: 32 fp32 values per thread in the butterflies
    if (d.gs < RUN || ROT) {
      if constexpr (RUN / 2 >= 32 && D / (RUN / 2) <= 4) chan_decode_any<T, D, RUN / 2, ROT>(p, d, tr.s, j0, rows, tile);
      else chan_decode_any<T, D, RUN, ROT>(p, d, tr.s, j0, rows, tile);
    } else {
      chan_decode_any<T, D, RUN, ROT>(p, d, tr.s, j0, rows, tile);
    }
  }
  __syncthreads();
  // the tile's rows leave as 16-byte vectors, 16 lanes per 256-byte row: thread =
  // (chunk, rows r0, r0 + STEP, ...)
  constexpr int CH = G::kRowBytes / 16, STEP = kDThreads / CH;
  const int c = threadIdx.x % CH, r0 = threadIdx.x / CH;
#pragma unroll
  for (int i = 0; i < kDTile / STEP; ++i) {
    const int r = r0 + i * STEP;
    const int t_out = r < rows ? toks[r] : -1;
    if (t_out >= 0)
      reinterpret_cast<uint4*>(out + (int64_t)t_out * D)[c] = *reinterpret_cast<const uint4*>(tile + r * G::kPitchB + c * 16);
  }
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
    T* out = reinterpret_cast<T*>(which ? p.out_v : p.out_k) + ((int64_t)s * p.out_T + tok) * D;
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
  const int64_t o = ((int64_t)s * p.out_T + tok) * p.D + c;
  reinterpret_cast<T*>(p.out_k)[o] = reinterpret_cast<const T*>(p.ret_k)[i];
  reinterpret_cast<T*>(p.out_v)[o] = reinterpret_cast<const T*>(p.ret_v)[i];
}

template <typename T, int D, int AXIS, bool ROT>
static cudaError_t launch_dq_variant(const DequantParams& p, int tensor, bool retained, bool standard, bool cold,
                                     cudaStream_t st) {
  using G = DGeom<T, D>;
  const DequantParams q = tiers_only(p, retained, standard, cold);
  const int64_t tiles = (int64_t)q.S * q.tiles_slice;
  if (tiles == 0) return cudaSuccess;
  const size_t sm = G::kTile + kDTile * sizeof(int);
  auto kern = dequantize_tile_kernel<T, D, AXIS, ROT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)tiles, kDThreads, sm, st>>>(q, tensor, retained ? 1 : 0);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_dq_tile(const DequantParams& p, cudaStream_t st, cudaStream_t st_rot) {
  if ((int64_t)p.S * p.tiles_slice == 0) return cudaSuccess;
  for (int tensor = 0; tensor < 2; ++tensor) {
    const int v1 = p.tiles[1] ? tier_variant(p.t[GKV_STD_K + tensor]) : -1;
    const int v2 = p.tiles[2] ? tier_variant(p.t[GKV_COLD_K + tensor]) : -1;
    bool retained = p.tiles[0] > 0;
    for (int v = 0; v < 4; ++v) {
      const bool standard = v1 == v, cold = v2 == v;
      const bool ret_here = retained && (standard || cold || (v1 < 0 && v2 < 0 && v == 2));
      if (!standard && !cold && !ret_here) continue;
      cudaError_t e;
      switch (v) {
        case 0: e = launch_dq_variant<T, D, GKV_AXIS_TOKEN, false>(p, tensor, ret_here, standard, cold, st); break;
        case 2: e = launch_dq_variant<T, D, GKV_AXIS_CHANNEL, false>(p, tensor, ret_here, standard, cold, st); break;
        case 3: e = launch_dq_variant<T, D, GKV_AXIS_CHANNEL, true>(p, tensor, ret_here, standard, cold, st_rot); break;
        default: e = cudaErrorInvalidConfiguration; break;  // rotated token axis: general path only
      }
      if (e != cudaSuccess) return e;
      if (ret_here) retained = false;
    }
  }
  return cudaSuccess;
}

template <typename T>
static cudaError_t launch_dq_tile_d(const DequantParams& p, cudaStream_t st, cudaStream_t st_rot) {
  if (p.D == 64) return launch_dq_tile<T, 64>(p, st, st_rot);
  if (p.D == 128) return launch_dq_tile<T, 128>(p, st, st_rot);
  return cudaErrorInvalidConfiguration;
}

// Rotated-tier launches on st_rot, the others on st (the caller orders the two
// streams).
cudaError_t launch_dequantize_tiles(const DequantParams& p, int dtype, cudaStream_t st, cudaStream_t st_rot) {
  if (dtype == GKV_BF16) return launch_dq_tile_d<__nv_bfloat16>(p, st, st_rot);
  if (dtype == GKV_F16) return launch_dq_tile_d<__half>(p, st, st_rot);
  return launch_dq_tile_d<float>(p, st, st_rot);
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
