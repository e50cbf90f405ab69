// Quantize + pack kernels (core.py:647-772, 848-910, 945-956, 979-990).
//
// Fast path: one launch per (tensor, kernel variant) -- for the graphkv profile
// keys, plain values and rotated cold values; one block of 128 threads per tile of
// 64 consecutive tier rows of one slice.  The threads gather the tile's
// rows into shared memory with 16-byte asynchronous copies, then quantize them,
// each thread holding whole quantization groups in registers:
//  - token-axis groups (K): a thread owns one 32-bit column word (two 16-bit
//    channels, or one fp32 channel) over the group's gs rows; lanes of a warp own
//    consecutive words of the same rows, so the column reads are conflict-free;
//  - channel-axis groups (V): a thread owns a run of 128 bytes of one row (a whole
//    group, or 1/2 or 1/4 of one, combined with the lanes 8 or 16 apart); the 8
//    lanes of a quarter-warp read 8 different rows, so the 16-byte reads are
//    conflict-free (row pitch = 4 words mod 32 banks).
// Rotated V rows (cold tier) are transformed in registers: butterflies inside the
// thread, then across the lanes that hold the rest of the row.  Group statistics
// use packed 16-bit min/max, the scale one fused quotient, the codes the packed
// quotient of gkv_common.cuh.  Retained rows are copied by tiles of the same launch.
//
// General path: any geometry the tiles do not cover (group sizes that are not
// 32 or 64 along tokens, group sizes that are not powers of two, padded head
// dims, tiny tiers, unaligned inputs): one thread per group computes the scale,
// one thread per output byte packs the codes.
#pragma once

#include <algorithm>

#include "gkv_params.cuh"

namespace gkv {

constexpr int kQThreads = 128;  // threads of a quantize tile block
constexpr int kQWarps = kQThreads / 32;
constexpr int kQRows = 32;      // rows of a token-axis column run (half a tile)
constexpr int kQTile = 64;      // tier rows of a quantize tile

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename T, int D>
struct QGeom {
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kPitchB = kRowBytes + 16;  // +16 B per row: consecutive rows start 4 banks apart
  static constexpr int kPitchW = kPitchB / 4;
  static constexpr int kWords = kRowBytes / 4;     // 32-bit words per row
  static constexpr int kChunks = kRowBytes / 16;   // 16-byte chunks per row
  static constexpr int kEPW = 4 / (int)sizeof(T);  // elements per word
  static constexpr int kRun = 128 / (int)sizeof(T);  // elements of a channel-axis run (128 bytes)
  static constexpr size_t kTileBytes = (size_t)kQTile * kPitchB;              // one tensor's tile
  static constexpr size_t kSmem = kTileBytes + (size_t)kWords * 2 * 2 * 4;   // + token-axis exchange
};

// ---------------------------------------------------------------------------
// retained rows
// ---------------------------------------------------------------------------
// Retained rows of one tensor: thread = (16-byte chunk, rows r0, r0 + STEP, ...);
// all of a thread's loads are issued before its stores.
template <typename T, int D>
__device__ void copy_retained_tile(const QuantParams& p, const T* src, int64_t st, void* ret, int gslice, int tile) {
  constexpr int kVec = 16 / (int)sizeof(T);
  constexpr int kChunks = D / kVec;
  constexpr int STEP = kQThreads / kChunks;
  constexpr int N = kRetTile / STEP;
  const int R = p.n_tier[0];
  const int j0 = tile * kRetTile;
  const int rows = min(kRetTile, R - j0);
  T* dst = reinterpret_cast<T*>(ret) + ((int64_t)gslice * R + j0) * D;
  const int c = threadIdx.x % kChunks, r0 = threadIdx.x / kChunks;
  uint4 v[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int r = r0 + i * STEP;
    v[i] = make_uint4(0u, 0u, 0u, 0u);
    if (r < rows) {
      int tok = p.idx[0][j0 + r];
      if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); tok = 0; }
      v[i] = ldg_stream(src + tok * st + c * kVec);
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int r = r0 + i * STEP;
    if (r < rows) *reinterpret_cast<uint4*>(dst + r * D + c * kVec) = v[i];
  }
}

// Hadamard rotation of the tile's rows in shared memory (token-axis tensors with
// the rotation), one warp per row.
template <typename T, int D>
__device__ void rotate_rows_smem(T* sx, float div, float inv, int hw) {
  using G = QGeom<T, D>;
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  for (int r = hw; r < kQTile; r += kQWarps) {
    T* row = reinterpret_cast<T*>(reinterpret_cast<uint8_t*>(sx) + r * G::kPitchB) + lane * EPL;
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = Elem<T>::to_f32(row[i]);
    fwht_warp<EPL>(v);
#pragma unroll
    for (int i = 0; i < EPL; ++i) row[i] = hadamard_scale<T>(v[i], div, inv);
  }
}

// ---------------------------------------------------------------------------
// encoding from data words
// ---------------------------------------------------------------------------
// Two consecutive elements (e, e + 1) of a run held as 32-bit data words.
template <typename T, int NW>
__device__ __forceinline__ uint64_t pair_at(const uint32_t (&w)[NW], int e) {
  if constexpr (sizeof(T) == 4) return pk2(__uint_as_float(w[e]), __uint_as_float(w[e + 1]));
  else return Word16<T>::pair(w[e >> 1]);
}

// Quotient, [zero point and clamp], magic add of a pair of elements.
template <bool AFF>
__device__ __forceinline__ uint64_t code_pair(uint64_t x2, uint64_t inv2, uint64_t nsc2, uint64_t zp2, uint64_t mg2,
                                              float hi) {
  uint64_t a2 = quot2(x2, nsc2, inv2);
  if (AFF) {
    a2 = add2(a2, zp2);
    a2 = pk2(fminf(fmaxf(lo2(a2), 0.f), hi), fminf(fmaxf(hi2(a2), 0.f), hi));
  }
  return add2(a2, mg2);
}

// Encode a run and store its codes in pieces of at most 16 bytes as they complete
// (keeps few code words live).  `store` false: encode only (lanes that hold
// padding rows still take part in the warp's shuffles but write nothing).
template <typename T, int SB, bool AFF, int NW>
__device__ __forceinline__ void encode_store_run(const uint32_t (&w)[NW], const FastCoder& c, uint8_t* dst,
                                                 bool store) {
  constexpr int N = NW * (4 / (int)sizeof(T));
  constexpr int EPC = 32 / SB;
  constexpr int NC = N / EPC;                 // code words of the run
  constexpr int PIECE = NC < 4 ? NC : 4;      // code words per store
  static_assert(N % EPC == 0 && NC % PIECE == 0, "whole code words");
  const uint64_t inv2 = pk2(c.inv, c.inv), nsc2 = pk2(-c.scale, -c.scale);
  const uint64_t mg2 = pk2(c.magic, c.magic), zp2 = pk2(c.zp, c.zp);
#pragma unroll
  for (int q0 = 0; q0 < NC; q0 += PIECE) {
    uint32_t out[PIECE];
#pragma unroll
    for (int q = 0; q < PIECE; ++q) {
      uint32_t acc = 0;
#pragma unroll
      for (int j = EPC / 2 - 1; j >= 0; --j) {
        const uint64_t t2 = code_pair<AFF>(pair_at<T>(w, (q0 + q) * EPC + 2 * j), inv2, nsc2, zp2, mg2, c.hi);
        acc = acc * (1u << SB) + hi32(t2);
        acc = acc * (1u << SB) + lo32(t2);
      }
      out[q] = (acc - magic_sum<SB>(EPC)) ^ (c.flip & slot_mask<SB>(EPC));
    }
    if (store) store_bytes<PIECE * 4>(dst + q0 * 4, out);
  }
}

// Same for two channels held in the halves of 16-bit column words.
template <typename T, int SB, bool AFF, int GS>
__device__ __forceinline__ void encode_store_columns(const uint32_t (&x)[GS], const FastCoder& c0,
                                                     const FastCoder& c1, uint8_t* dst0, uint8_t* dst1) {
  constexpr int EPC = 32 / SB;
  constexpr int NC = GS / EPC;
  constexpr int PIECE = NC < 4 ? NC : 4;
  const uint64_t inv2 = pk2(c0.inv, c1.inv), nsc2 = pk2(-c0.scale, -c1.scale);
  const uint64_t mg2 = pk2(c0.magic, c1.magic), zp2 = pk2(c0.zp, c1.zp);
#pragma unroll
  for (int q0 = 0; q0 < NC; q0 += PIECE) {
    uint32_t o0[PIECE], o1[PIECE];
#pragma unroll
    for (int q = 0; q < PIECE; ++q) {
      uint32_t a0 = 0, a1 = 0;
#pragma unroll
      for (int i = EPC - 1; i >= 0; --i) {
        const uint64_t t2 = code_pair<AFF>(Word16<T>::pair(x[(q0 + q) * EPC + i]), inv2, nsc2, zp2, mg2, c0.hi);
        a0 = a0 * (1u << SB) + lo32(t2);
        a1 = a1 * (1u << SB) + hi32(t2);
      }
      o0[q] = (a0 - magic_sum<SB>(EPC)) ^ (c0.flip & slot_mask<SB>(EPC));
      o1[q] = (a1 - magic_sum<SB>(EPC)) ^ (c1.flip & slot_mask<SB>(EPC));
    }
    store_bytes<PIECE * 4>(dst0 + q0 * 4, o0);
    store_bytes<PIECE * 4>(dst1 + q0 * 4, o1);
  }
}

// Statistics of a run of data words: absmax (symmetric) or min/max (affine),
// per element half for 16-bit types.
template <typename T, bool AFF, int NW>
__device__ __forceinline__ void run_stats(const uint32_t (&w)[NW], float& mn, float& mx) {
  if constexpr (sizeof(T) == 4) {
    mn = __int_as_float(0x7f800000);
    mx = AFF ? -__int_as_float(0x7f800000) : 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const float f = __uint_as_float(w[i]);
      if (AFF) { mn = fminf(mn, f); mx = fmaxf(mx, f); }
      else mx = fmaxf(mx, fabsf(f));
    }
  } else {
    using W = Word16<T>;
    if (AFF) {
      uint32_t a = W::kPosInf, b = W::kNegInf;
#pragma unroll
      for (int i = 0; i < NW; ++i) { a = W::vmin(a, w[i]); b = W::vmax(b, w[i]); }
      mn = fminf(W::lo(a), W::hi(a));
      mx = fmaxf(W::lo(b), W::hi(b));
    } else {
      uint32_t a = 0u;
#pragma unroll
      for (int i = 0; i < NW; ++i) a = W::amax(a, w[i]);
      a &= 0x7FFF7FFFu;
      mn = 0.f;
      mx = fmaxf(W::lo(a), W::hi(a));
    }
  }
}

// ---------------------------------------------------------------------------
// token-axis groups (K): thread = (column word, run of 32 rows)
// ---------------------------------------------------------------------------
// Statistics of a column run as 32-bit words: 16-bit types keep both channels
// packed (absmax, or min and max); fp32 keeps the float bits.
template <typename T, bool AFF>
struct ColStats {
  uint32_t a, b;  // symmetric: a = absmax; affine: a = min, b = max
  __device__ __forceinline__ void init() {
    if constexpr (sizeof(T) == 4) {
      a = AFF ? 0x7f800000u : 0u;
      b = 0xff800000u;
    } else {
      a = AFF ? Word16<T>::kPosInf : 0u;
      b = Word16<T>::kNegInf;
    }
  }
  __device__ __forceinline__ void add(uint32_t x) {
    if constexpr (sizeof(T) == 4) {
      const float f = __uint_as_float(x);
      if (AFF) {
        a = __float_as_uint(fminf(__uint_as_float(a), f));
        b = __float_as_uint(fmaxf(__uint_as_float(b), f));
      } else {
        a = __float_as_uint(fmaxf(__uint_as_float(a), fabsf(f)));
      }
    } else {
      if (AFF) { a = Word16<T>::vmin(a, x); b = Word16<T>::vmax(b, x); }
      else a = Word16<T>::amax(a, x);
    }
  }
  __device__ __forceinline__ void merge(const ColStats& o) {
    if constexpr (sizeof(T) == 4) {
      if (AFF) {
        a = __float_as_uint(fminf(__uint_as_float(a), __uint_as_float(o.a)));
        b = __float_as_uint(fmaxf(__uint_as_float(b), __uint_as_float(o.b)));
      } else {
        a = __float_as_uint(fmaxf(__uint_as_float(a), __uint_as_float(o.a)));
      }
    } else {
      if (AFF) { a = Word16<T>::vmin(a, o.a); b = Word16<T>::vmax(b, o.b); }
      else a = Word16<T>::amax(a, o.a);
    }
  }
};

// Tile rows are split into two runs of 32 (thread = (word w, run h)); lanes of a
// warp own consecutive words of the same rows.  A 64-row group spans both runs:
// their statistics meet through shared memory (`xch`, 2 words per item).
template <typename T, int D, int GS, int SB, bool AFF>
__device__ void quant_tokens(const TensorDesc& d, const uint8_t* sx, int gslice, int j0, uint32_t* xch) {
  using G = QGeom<T, D>;
  constexpr int NH = kQTile / kQRows;          // runs per column
  constexpr int ITEMS = G::kWords * NH;
  constexpr bool SPLIT = GS > kQRows;          // a group spans the two runs
  static_assert(GS == 32 || GS == 64, "token-axis groups of 32 or 64 rows");
  constexpr int CPW = 4 / (int)sizeof(T);
  for (int base = 0; base < ITEMS; base += kQThreads) {  // uniform trip count: barriers inside
    const int item = base + (int)threadIdx.x;
    const bool act = item < ITEMS;
    const int h = act ? item / G::kWords : 0, w = act ? item - h * G::kWords : 0;
    const int tok0 = j0 + h * kQRows;            // first tier row of this run
    const uint32_t* col = reinterpret_cast<const uint32_t*>(sx + (h * kQRows) * G::kPitchB) + w;
    uint32_t x[kQRows];
#pragma unroll
    for (int i = 0; i < kQRows; ++i) x[i] = act ? col[i * G::kPitchW] : 0u;
    ColStats<T, AFF> cs;
    cs.init();
#pragma unroll
    for (int i = 0; i < kQRows; ++i) cs.add(x[i]);
    if constexpr (SPLIT) {
      if (act) { xch[2 * item] = cs.a; xch[2 * item + 1] = cs.b; }
      __syncthreads();
      if (act) {
        const int other = (h ^ 1) * G::kWords + w;
        ColStats<T, AFF> o;
        o.a = xch[2 * other];
        o.b = xch[2 * other + 1];
        cs.merge(o);
      }
      __syncthreads();  // xch is reused by the next round
    }
    if (!act || tok0 >= d.n_pad) continue;
    const bool first = (h * kQRows) % GS == 0;   // this run starts its group: it stores the scales
    const int gtok = tok0 - (h * kQRows) % GS;
    constexpr int NB = kQRows * SB / 8;          // code bytes per channel and run
    if constexpr (CPW == 1) {
      const float mn = __uint_as_float(cs.a), mx = AFF ? __uint_as_float(cs.b) : __uint_as_float(cs.a);
      const FastCoder c = AFF ? aff_coder(mn, mx, d.qmax, d.rqmax)
                              : sym_coder(mx, d.qmax, d.rqmax, d.bits, d.packed != 0);
      const int ch = w;
      if (first) {
        const int64_t gi = ((int64_t)gslice * D + ch) * d.groups_row + (gtok >> d.log2gs);
        store_scale(d.scales, gi, d.scale_dtype, c.scale);
        if (AFF) d.zps[gi] = (uint8_t)c.zp;
      }
      const int64_t e0 = ((int64_t)gslice * D + ch) * d.n_pad + tok0;
      encode_store_run<T, SB, AFF, kQRows>(x, c, d.codes + (e0 * SB) / 8, true);
      (void)NB;
    } else {
      using W = Word16<T>;
      FastCoder c0, c1;
      if (AFF) {
        c0 = aff_coder(W::lo(cs.a), W::lo(cs.b), d.qmax, d.rqmax);
        c1 = aff_coder(W::hi(cs.a), W::hi(cs.b), d.qmax, d.rqmax);
      } else {
        const uint32_t am = cs.a & 0x7FFF7FFFu;
        c0 = sym_coder(W::lo(am), d.qmax, d.rqmax, d.bits, d.packed != 0);
        c1 = sym_coder(W::hi(am), d.qmax, d.rqmax, d.bits, d.packed != 0);
      }
      const int ch = 2 * w;
      if (first) {
        const int64_t gi0 = ((int64_t)gslice * D + ch) * d.groups_row + (gtok >> d.log2gs);
        store_scale(d.scales, gi0, d.scale_dtype, c0.scale);
        store_scale(d.scales, gi0 + d.groups_row, d.scale_dtype, c1.scale);
        if (AFF) {
          d.zps[gi0] = (uint8_t)c0.zp;
          d.zps[gi0 + d.groups_row] = (uint8_t)c1.zp;
        }
      }
      const int64_t e0 = ((int64_t)gslice * D + ch) * d.n_pad + tok0;
      encode_store_columns<T, SB, AFF, kQRows>(x, c0, c1, d.codes + (e0 * SB) / 8, d.codes + ((e0 + d.n_pad) * SB) / 8);
    }
  }
}

// ---------------------------------------------------------------------------
// channel-axis groups (V): thread = (row, run of 128 bytes)
// ---------------------------------------------------------------------------
template <typename T, int NW>
__device__ __forceinline__ void load_run(const uint8_t* src, uint32_t (&w)[NW]) {
#pragma unroll
  for (int q = 0; q < NW / 4; ++q) {
    const uint4 r = reinterpret_cast<const uint4*>(src)[q];
    w[4 * q] = r.x; w[4 * q + 1] = r.y; w[4 * q + 2] = r.z; w[4 * q + 3] = r.w;
  }
}

template <typename T, int RUN, int NW>
__device__ __forceinline__ void words_to_pairs(const uint32_t (&w)[NW], uint64_t (&v)[RUN / 2]) {
#pragma unroll
  for (int k = 0; k < RUN / 2; ++k) v[k] = pair_at<T>(w, 2 * k);
}

template <typename T, int RUN, int NW>
__device__ __forceinline__ void pairs_to_words(const uint64_t (&v)[RUN / 2], uint32_t (&w)[NW]) {
#pragma unroll
  for (int k = 0; k < RUN / 2; ++k) {
    if constexpr (sizeof(T) == 4) {
      w[2 * k] = lo32(v[k]);
      w[2 * k + 1] = hi32(v[k]);
    } else {
      w[k] = Word16<T>::round2(lo2(v[k]), hi2(v[k]));
    }
  }
}

// ---------------------------------------------------------------------------
// Rotated channel-axis groups of 16-bit rows of 128 elements (the long-context
// cold value tier): two threads per row, thread u (lane bit 3) holding elements
// 64u .. 64u + 63 as 32 packed fp32 pairs (element 2m, 2m + 1 in pair m).
//  - Stages h = 1 .. 32 (core.py:950-955) run in the thread: h = 1 inside a pair,
//    h >= 2 between pairs.  Thread 1 holds its halves swapped (pair m <-> m ^ 16)
//    so that both threads hand over pairs 16 .. 31 below; its h = 32 butterfly
//    writes the sum to the pair that holds the lower element, through a signed
//    fused multiply-add that rounds like the add / subtract.
//  - Stage h = 64 pairs element e of the two halves: each thread writes the 32
//    values it hands over as fp32 into its own 128 bytes of the staged row
//    (already in registers) and reads the partner's; thread 0 then computes
//    outputs 0..31 and 64..95, thread 1 outputs 32..63 and 96..127 (its
//    differences come out negated and are flipped after rounding -- division and
//    rounding are sign-symmetric).
//  - Then y / sqrt(128) (fused quotient when proven exact: every input of the
//    warp's rows is +0 or at least 2^-88 in magnitude, so no output is -0 or
//    below 2^-99; IEEE division otherwise), the cast to the input dtype, group
//    statistics (two groups of 64 or one of 128) and the codes.
//  - int2 symmetric codes of 16-bit values: q = round(y / s) with |y| <= s takes
//    one fused multiply-add y * inv + magic with inv = fl(1 / s) * (1 - 2^-16):
//    distinct 16-bit values differ by at least 2^-11 relative, so y / s is 0.5
//    exactly (a tie, rounded to 0 by the reference) or at least 2^-12 away from
//    it, and the product stays on the same side of 0.5 as the exact quotient.
// ---------------------------------------------------------------------------
template <int SB, bool AFF, int NW, typename T>
__device__ __forceinline__ void encode_int2_sym16(const uint32_t (&w)[NW], float inv_lo, uint8_t* dst, bool store) {
  static_assert(SB == 2 && NW == 16, "32 int2 codes");
  const uint64_t inv2 = pk2(inv_lo, inv_lo);
  const float mg = kMagic + 2.f;
  const uint64_t mg2 = pk2(mg, mg);
  uint32_t out[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {  // 16 codes per 32-bit word
    uint32_t acc = 0;
#pragma unroll
    for (int j = 7; j >= 0; --j) {
      const uint64_t t2 = fma2(Word16<T>::pair(w[8 * q + j]), inv2, mg2);
      acc = acc * 4u + hi32(t2);
      acc = acc * 4u + lo32(t2);
    }
    out[q] = acc - magic_sum<2>(16);
  }
  if (store) store_bytes<8>(dst, out);
}

template <typename T, int SB, bool AFF>
__device__ void quant_rot_pair(const TensorDesc& d, uint8_t* sx, int gslice, int j0, int rows, int ht, float div,
                               float rdiv, bool fused_ok) {
  using G = QGeom<T, 128>;
  using W = Word16<T>;
  constexpr int ROWS_STEP = 16;
  constexpr int STEPS = kQTile / ROWS_STEP;
  const int lane = ht & 31, hw = ht >> 5;
  const int j = lane & 7, k = lane >> 3;
  const int u = k & 1, rb = k >> 1;
  const float sg = u ? -1.f : 1.f;
  const uint64_t sgp = pk2(sg, sg), sgn = pk2(-sg, -sg);
#pragma unroll 1
  for (int step = hw; step < STEPS; step += kQWarps) {
    const int r = step * ROWS_STEP + rb * 8 + j;
    uint8_t* own = sx + r * G::kPitchB + u * 128;
    uint64_t v[32];
    uint32_t lowest = W::kMaxFinite;  // packed magnitude minimum of the inputs
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      // thread 1 takes its two 32-element halves in swapped order
      const uint4 a = reinterpret_cast<const uint4*>(own)[u ? (q ^ 4) : q];
      const uint32_t wq[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        lowest = W::amin(lowest, wq[i]);
        const float x0 = W::lo(wq[i]), x1 = W::hi(wq[i]);
        v[4 * q + i] = pk2(__fadd_rn(x0, x1), __fsub_rn(x0, x1));  // h = 1
      }
    }
    // h = 2 .. 16: pairs m and m + h/2 (inside each half of 16 pairs)
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
    // h = 32: pairs m and m + 16 (thread 1: lower element in m + 16)
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const uint64_t a = v[m], b = v[m + 16];
      v[m] = fma2(sgp, a, b);
      v[m + 16] = fma2(sgn, b, a);
    }
    // Outputs are sums of multiples of the smallest input's unit in the last
    // place, so with every input at least 2^-88 in magnitude no output is below
    // 2^-95 (quotient >= 2^-99) and none is -0: the fused quotient is exact.
    // Rows with a zero or tiny input divide exactly (whole warp).
    const uint32_t mag = lowest & 0x7FFF7FFFu;
    const bool small = !(fminf(W::lo(mag), W::hi(mag)) >= 3.2311742677852644e-27f /* 2^-88 */);
    const bool fused = fused_ok && !__any_sync(kFull, small);
    // hand over pairs 16 .. 31 through the thread's own (consumed) 128 bytes
    uint4* mine = reinterpret_cast<uint4*>(own);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      mine[q] = make_uint4(lo32(v[16 + 2 * q]), hi32(v[16 + 2 * q]), lo32(v[17 + 2 * q]), hi32(v[17 + 2 * q]));
    __syncwarp();
    const uint4* theirs = reinterpret_cast<const uint4*>(sx + r * G::kPitchB + (u ^ 1) * 128);
    uint32_t ws[16], wd[16];  // rounded outputs: sums (group of the lower half), differences
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 t = theirs[q];
      const uint64_t o0 = pk2u(t.x, t.y), o1 = pk2u(t.z, t.w);
      uint64_t s0 = add2(v[2 * q], o0), s1 = add2(v[2 * q + 1], o1);
      uint64_t d0 = sub2(v[2 * q], o0), d1 = sub2(v[2 * q + 1], o1);
      if (fused) {
        const uint64_t nd2 = pk2(-div, -div), rd2 = pk2(rdiv, rdiv);
        s0 = quot2(s0, nd2, rd2);
        s1 = quot2(s1, nd2, rd2);
        d0 = quot2(d0, nd2, rd2);
        d1 = quot2(d1, nd2, rd2);
      } else {
        s0 = pk2(__fdiv_rn(lo2(s0), div), __fdiv_rn(hi2(s0), div));
        s1 = pk2(__fdiv_rn(lo2(s1), div), __fdiv_rn(hi2(s1), div));
        d0 = pk2(__fdiv_rn(lo2(d0), div), __fdiv_rn(hi2(d0), div));
        d1 = pk2(__fdiv_rn(lo2(d1), div), __fdiv_rn(hi2(d1), div));
      }
      ws[2 * q] = W::round2(lo2(s0), hi2(s0));
      ws[2 * q + 1] = W::round2(lo2(s1), hi2(s1));
      wd[2 * q] = W::round2(lo2(d0), hi2(d0));
      wd[2 * q + 1] = W::round2(lo2(d1), hi2(d1));
    }
    const uint32_t flip = u ? 0x80008000u : 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) wd[i] ^= flip;
    // statistics of the two groups (sums: elements 0..63, differences: 64..127)
    float mn0, mx0, mn1, mx1;
    run_stats<T, AFF, 16>(ws, mn0, mx0);
    run_stats<T, AFF, 16>(wd, mn1, mx1);
    mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 8));
    mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 8));
    if (AFF) {
      mn0 = fminf(mn0, __shfl_xor_sync(kFull, mn0, 8));
      mn1 = fminf(mn1, __shfl_xor_sync(kFull, mn1, 8));
    }
    if (d.gs == 128) {
      mx0 = mx1 = fmaxf(mx0, mx1);
      mn0 = mn1 = fminf(mn0, mn1);
    }
    const FastCoder c0 = AFF ? aff_coder(mn0, mx0, d.qmax, d.rqmax) : sym_coder(mx0, d.qmax, d.rqmax, d.bits, d.packed != 0);
    const FastCoder c1 = AFF ? aff_coder(mn1, mx1, d.qmax, d.rqmax) : sym_coder(mx1, d.qmax, d.rqmax, d.bits, d.packed != 0);
    const bool act = r < rows;
    const int64_t row = (int64_t)gslice * d.n + j0 + r;
    if (act) {
      if (d.gs == 128) {
        if (u == 0) {
          store_scale(d.scales, row, d.scale_dtype, c0.scale);
          if (AFF) d.zps[row] = (uint8_t)c0.zp;
        }
      } else {
        const FastCoder& c = u ? c1 : c0;
        store_scale(d.scales, row * 2 + u, d.scale_dtype, c.scale);
        if (AFF) d.zps[row * 2 + u] = (uint8_t)c.zp;
      }
    }
    uint8_t* codes = d.codes + ((row * d.n_pad) * SB) / 8;
    uint8_t* dst0 = codes + (32 * u * SB) / 8;          // sums: elements 32u .. 32u + 31
    uint8_t* dst1 = codes + ((64 + 32 * u) * SB) / 8;   // differences: 64 + 32u ..
    if constexpr (SB == 2 && !AFF) {
      // the one-FMA coder needs |y| <= s with s a 16-bit value (s >= 1e-8)
      const bool fast = d.packed && !(mx0 < kEps) && !(mx1 < kEps);
      if (fast) {
        const float k16 = 0.9999847412109375f;  // 1 - 2^-16
        encode_int2_sym16<2, false, 16, T>(ws, __fmul_rn(c0.inv, k16), dst0, act);
        encode_int2_sym16<2, false, 16, T>(wd, __fmul_rn(c1.inv, k16), dst1, act);
        continue;
      }
    }
    encode_store_run<T, SB, AFF, 16>(ws, c0, dst0, act);
    encode_store_run<T, SB, AFF, 16>(wd, c1, dst1, act);
  }
}

template <typename T, int D, int RUN, int SB, bool AFF, bool ROT>
__device__ void quant_channels(const TensorDesc& d, uint8_t* sx, int gslice, int j0, int rows, int ht,
                               float div, float rdiv, bool fused) {
  if constexpr (ROT && D == 128 && RUN == 64 && sizeof(T) == 2) {
    quant_rot_pair<T, SB, AFF>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
    return;
  }
  using G = QGeom<T, D>;
  constexpr int RPR = D / RUN;             // runs per row (1, 2 or 4)
  constexpr int NW = RUN * (int)sizeof(T) / 4;
  constexpr int ROWS_STEP = 32 / RPR;      // rows per warp step (lane = row j + 8 * (run + RPR * row block))
  constexpr int STEPS = kQTile / ROWS_STEP;
  static_assert(RPR == 1 || RPR == 2 || RPR == 4, "runs per row");
  const int lane = threadIdx.x & 31, hw = ht >> 5;
  const int j = lane & 7, k = lane >> 3;
  const int u = k % RPR, rb = k / RPR;
  const int rpg = d.gs / RUN;              // runs per group: 1, 2 or 4 (gs >= RUN)
#pragma unroll 1
  for (int step = hw; step < STEPS; step += kQWarps) {
    const int r = step * ROWS_STEP + rb * 8 + j;
    const uint8_t* src = sx + r * G::kPitchB + u * (RUN * (int)sizeof(T));
    uint32_t w[NW];
    load_run<T, NW>(src, w);
    if constexpr (ROT) {
      uint64_t v[RUN / 2];
      words_to_pairs<T, RUN, NW>(w, v);
      rotate_run<RUN, RPR>(v, u, div, rdiv, fused);
      pairs_to_words<T, RUN, NW>(v, w);
    }
    float mn, mx;
    run_stats<T, AFF, NW>(w, mn, mx);
    for (int m = 1; m < rpg; m <<= 1) {
      if (AFF) mn = fminf(mn, __shfl_xor_sync(kFull, mn, 8 * m));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8 * m));
    }
    const FastCoder c = AFF ? aff_coder(mn, mx, d.qmax, d.rqmax) : sym_coder(mx, d.qmax, d.rqmax, d.bits, d.packed != 0);
    const bool act = r < rows;
    const int64_t row = (int64_t)gslice * d.n + j0 + r;
    if (act && u % rpg == 0) {
      const int64_t gi = row * d.groups_row + u / rpg;
      store_scale(d.scales, gi, d.scale_dtype, c.scale);
      if (AFF) d.zps[gi] = (uint8_t)c.zp;
    }
    const int64_t e0 = row * d.n_pad + u * RUN;
    encode_store_run<T, SB, AFF, NW>(w, c, d.codes + (e0 * SB) / 8, act);
  }
}

// ---------------------------------------------------------------------------
// dispatch on the tensor's runtime parameters
// ---------------------------------------------------------------------------
template <typename T, int D, int SB>
__device__ __forceinline__ void quant_tile_tokens_sb(const TensorDesc& d, const uint8_t* sx, int gslice, int j0,
                                                     uint32_t* xch) {
  const bool aff = d.quantizer == GKV_AFFINE;
  if (d.gs == 64) {
    if (aff) quant_tokens<T, D, 64, SB, true>(d, sx, gslice, j0, xch);
    else quant_tokens<T, D, 64, SB, false>(d, sx, gslice, j0, xch);
  } else {
    if (aff) quant_tokens<T, D, 32, SB, true>(d, sx, gslice, j0, xch);
    else quant_tokens<T, D, 32, SB, false>(d, sx, gslice, j0, xch);
  }
}

template <typename T, int D, int RUN, int SB, bool ROT>
__device__ __forceinline__ void quant_tile_channels_sb(const TensorDesc& d, uint8_t* sx, int gslice, int j0,
                                                       int rows, int ht, float div, float rdiv, bool fused) {
  if (d.quantizer == GKV_AFFINE) quant_channels<T, D, RUN, SB, true, ROT>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
  else quant_channels<T, D, RUN, SB, false, ROT>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
}

template <typename T, int D, bool ROT>
__device__ __forceinline__ void quant_tile_channels(const TensorDesc& d, uint8_t* sx, int gslice, int j0,
                                                    int rows, int ht, float div, float rdiv, bool fused) {
  // run = 128 bytes, or half of that when the group is smaller
  constexpr int RUN = QGeom<T, D>::kRun;
  if (d.gs < RUN) {
    if constexpr (RUN / 2 >= 32 && D / (RUN / 2) <= 4) {
      if (d.sbits == 4) quant_tile_channels_sb<T, D, RUN / 2, 4, ROT>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
      else if (d.sbits == 2) quant_tile_channels_sb<T, D, RUN / 2, 2, ROT>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
      else quant_tile_channels_sb<T, D, RUN / 2, 8, ROT>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
    }
  } else {
    if (d.sbits == 4) quant_tile_channels_sb<T, D, RUN, 4, ROT>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
    else if (d.sbits == 2) quant_tile_channels_sb<T, D, RUN, 2, ROT>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
    else quant_tile_channels_sb<T, D, RUN, 8, ROT>(d, sx, gslice, j0, rows, ht, div, rdiv, fused);
  }
}

// Tile t of a launch -> (slice, tier, tile within the tier); tier 0 = retained rows.
struct TileRef {
  int s, tier, k;
};
__device__ __forceinline__ TileRef tile_ref(const QuantParams& p, int t) {
  TileRef r;
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

// Staging of a tile of one tensor with 16-byte asynchronous copies: thread =
// (chunk c, rows r0, r0 + STEP, ...), so the lanes of a warp cover whole rows
// (coalesced).  The rows' token indices are loaded one tile ahead, one per lane
// (tile_tokens), and handed out with shuffles when the copies are issued
// (stage_tile), so issuing never waits for a load.  Rows past the end of the
// tier are zero-filled (token-axis groups quantize them as padding).
template <typename T, int D>
struct StageMap {
  using G = QGeom<T, D>;
  static constexpr int STEP = kQThreads / G::kChunks;  // rows per pass of the block
  static constexpr int LPR = G::kChunks;               // lanes per row within a pass
  static constexpr int RPW = 32 / LPR;                 // rows of one pass held by a warp
  static constexpr int NPASS = kQTile / STEP;          // passes
  static_assert(LPR <= 32 && 32 % LPR == 0 && NPASS * RPW <= 32, "one index per lane");
};

template <typename T, int D>
__device__ __forceinline__ int tile_tokens(const QuantParams& p, const TileRef& tr) {
  using M = StageMap<T, D>;
  const int j0 = tr.k * kQTile;
  const int rows = min(kQTile, p.n_tier[tr.tier] - j0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // lane l holds the index of row (l / RPW) * STEP + warp * RPW + l % RPW
  const int lrow = (lane / M::RPW) * M::STEP + warp * M::RPW + lane % M::RPW;
  int tok = 0;
  if (lane < M::NPASS * M::RPW && lrow < rows) {
    tok = p.idx[tr.tier][j0 + lrow];
    if ((unsigned)tok >= (unsigned)p.T) { raise_error(kErrBadIndex); tok = 0; }
  }
  return tok;
}

template <typename T, int D>
__device__ __forceinline__ void stage_tile(const QuantParams& p, const TileRef& tr, const T* base, int64_t st,
                                           uint8_t* sx, int ltok) {
  using G = QGeom<T, D>;
  using M = StageMap<T, D>;
  const int j0 = tr.k * kQTile;
  const int rows = min(kQTile, p.n_tier[tr.tier] - j0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = threadIdx.x % M::LPR, b = lane / M::LPR;  // row of a pass: pass * STEP + warp * RPW + b
  const uint8_t* src0 = reinterpret_cast<const uint8_t*>(base) + c * 16;
  uint8_t* dst0 = sx + (warp * M::RPW + b) * G::kPitchB + c * 16;
#pragma unroll
  for (int i = 0; i < M::NPASS; ++i) {
    const int r = i * M::STEP + warp * M::RPW + b;
    const int tok = __shfl_sync(kFull, ltok, i * M::RPW + b);
    cp_async16(dst0 + i * M::STEP * G::kPitchB, src0 + (int64_t)tok * st * (int64_t)sizeof(T), r < rows ? 16u : 0u);
  }
}

// Slice base pointer and token stride of one tensor.
template <typename T>
__device__ __forceinline__ const T* tensor_base(const QuantParams& p, int s, int tensor, int64_t& st) {
  const LayerDesc& L = p.layers[find_layer(p, s)];
  const int local = s - L.slice_begin;
  const int b = p.layer_div.d ? (int)p.head_div.div((uint32_t)local) : local / L.heads;
  const int h = local - b * L.heads;
  st = tensor ? L.vs[2] : L.ks[2];
  return tensor ? reinterpret_cast<const T*>(L.v) + b * L.vs[0] + h * L.vs[1]
                : reinterpret_cast<const T*>(L.k) + b * L.ks[0] + h * L.ks[1];
}

// Does this launch handle tile t, and does it stage rows for it?
template <int AXIS>
__device__ __forceinline__ int tile_role(const QuantParams& p, const TileRef& tr, int tensor, int copy_retained) {
  if (tr.tier == 0) return copy_retained ? 1 : 0;  // 1: retained copy
  const TensorDesc& d = p.t[(tr.tier == 1 ? GKV_STD_K : GKV_COLD_K) + tensor];
  return d.axis == AXIS ? 2 : 0;                     // 2: quantize
}

// One block per tile of one tensor (`tensor` 1: values, 0: keys).  Compiled per
// grouping axis (AXIS) and rotation (ROT), so that each variant keeps only the
// registers it needs; a launch covers the tiers that use its variant (the host
// zeroes the tile counts of the others) and the retained rows when `copy_retained`.
// Many small blocks per SM: while some wait for their rows, others compute.
// INT2: the launch's rotated tiers are all packed int2 symmetric with groups of
// 64 or 128 (16-bit rows of 128): only that coder is compiled, which keeps the
// variant at 64 registers.
template <typename T, int D, int AXIS, bool ROT, bool INT2 = false>
__global__ void __launch_bounds__(kQThreads, INT2 ? 7 : sizeof(T) == 4 ? (AXIS == GKV_AXIS_TOKEN ? 7 : (ROT ? 5 : 7)) : (AXIS == GKV_AXIS_TOKEN ? 8 : (ROT ? 5 : 10)))
    quantize_tile_kernel(const __grid_constant__ QuantParams p, int tensor, int copy_retained) {
  extern __shared__ __align__(128) uint8_t smem[];
  using G = QGeom<T, D>;
  const TileRef tr = tile_ref(p, blockIdx.x);
  const int role = tile_role<AXIS>(p, tr, tensor, copy_retained);
  if (role == 0) return;
  const TensorDesc& d = p.t[(tr.tier == 1 ? GKV_STD_K : GKV_COLD_K) + tensor];
  if (role == 2 && (d.rotation != 0) != ROT) return;  // not this variant's tier
  const int gslice = p.slice_offset + tr.s;
  int64_t st;
  const T* base = tensor_base<T>(p, tr.s, tensor, st);
  if (role == 1) {
    copy_retained_tile<T, D>(p, base, st, tensor ? p.ret_v : p.ret_k, gslice, tr.k);
    return;
  }
  stage_tile<T, D>(p, tr, base, st, smem, tile_tokens<T, D>(p, tr));
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  const int j0 = tr.k * kQTile;
  if constexpr (AXIS == GKV_AXIS_TOKEN) {
    if constexpr (ROT) {
      rotate_rows_smem<T, D>(reinterpret_cast<T*>(smem), p.had_div, p.had_inv, threadIdx.x >> 5);
      __syncthreads();
    }
    uint32_t* xch = reinterpret_cast<uint32_t*>(smem + G::kTileBytes);
    if (d.sbits == 4) quant_tile_tokens_sb<T, D, 4>(d, smem, gslice, j0, xch);
    else if (d.sbits == 2) quant_tile_tokens_sb<T, D, 2>(d, smem, gslice, j0, xch);
    else quant_tile_tokens_sb<T, D, 8>(d, smem, gslice, j0, xch);
  } else {
    const int rows = min(kQTile, p.n_tier[tr.tier] - j0);
    if constexpr (INT2) {
      quant_channels<T, D, 64, 2, false, true>(d, smem, gslice, j0, rows, threadIdx.x, p.had_div, p.had_inv,
                                               p.had_fused != 0);
    } else {
      quant_tile_channels<T, D, ROT>(d, smem, gslice, j0, rows, threadIdx.x, p.had_div, p.had_inv,
                                     p.had_fused != 0);
    }
  }
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

// Per tensor (keys, values): one launch per kernel variant its tiers need; the
// first of them also copies the tensor's retained rows.
// Packed int2 symmetric tensor with groups of 64 or 128 along 16-bit rows of 128.
inline bool int2_rot_tensor(const TensorDesc& d, int esize, int D) {
  return esize == 2 && D == 128 && d.bits == 2 && d.quantizer == GKV_SYMMETRIC && d.packed &&
         d.axis == GKV_AXIS_CHANNEL && d.rotation && (d.gs == 64 || d.gs == 128);
}

template <typename T, int D, int AXIS, bool ROT, bool INT2 = false>
static cudaError_t launch_variant(const QuantParams& p, int tensor, bool retained, bool standard, bool cold,
                                  cudaStream_t st) {
  const QuantParams q = tiers_only(p, retained, standard, cold);
  const int64_t tiles = (int64_t)q.S * q.tiles_slice;
  if (tiles == 0) return cudaSuccess;
  const size_t sm = QGeom<T, D>::kSmem;
  auto kern = quantize_tile_kernel<T, D, AXIS, ROT, INT2>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)tiles, kQThreads, sm, st>>>(q, tensor, retained ? 1 : 0);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_tile(const QuantParams& p, cudaStream_t st, cudaStream_t st_rot) {
  if ((int64_t)p.S * p.tiles_slice == 0) return cudaSuccess;
  for (int tensor = 0; tensor < 2; ++tensor) {
    const int v1 = p.tiles[1] ? tier_variant(p.t[GKV_STD_K + tensor]) : -1;
    const int v2 = p.tiles[2] ? tier_variant(p.t[GKV_COLD_K + tensor]) : -1;
    bool retained = p.tiles[0] > 0;  // copied by the first launch of this tensor
    for (int v = 0; v < 4; ++v) {
      const bool standard = v1 == v, cold = v2 == v;
      const bool ret_here = retained && (standard || cold || (v1 < 0 && v2 < 0 && v == 2));
      if (!standard && !cold && !ret_here) continue;
      cudaError_t e;
      switch (v) {
        case 0: e = launch_variant<T, D, GKV_AXIS_TOKEN, false>(p, tensor, ret_here, standard, cold, st); break;
        case 1: e = launch_variant<T, D, GKV_AXIS_TOKEN, true>(p, tensor, ret_here, standard, cold, st); break;
        case 2: e = launch_variant<T, D, GKV_AXIS_CHANNEL, false>(p, tensor, ret_here, standard, cold, st); break;
        default: {
          const bool int2 = (!standard || int2_rot_tensor(p.t[GKV_STD_K + tensor], sizeof(T), D)) &&
                            (!cold || int2_rot_tensor(p.t[GKV_COLD_K + tensor], sizeof(T), D));
          if constexpr (sizeof(T) == 2 && D == 128) {
            if (int2) {
              e = launch_variant<T, D, GKV_AXIS_CHANNEL, true, true>(p, tensor, ret_here, standard, cold, st_rot);
              break;
            }
          }
          e = launch_variant<T, D, GKV_AXIS_CHANNEL, true>(p, tensor, ret_here, standard, cold, st_rot);
          break;
        }
      }
      if (e != cudaSuccess) return e;
      if (ret_here) retained = false;
    }
  }
  return cudaSuccess;
}

template <typename T>
static cudaError_t launch_tile_d(const QuantParams& p, cudaStream_t st, cudaStream_t st_rot) {
  if (p.D == 64) return launch_tile<T, 64>(p, st, st_rot);
  if (p.D == 128) return launch_tile<T, 128>(p, st, st_rot);
  return cudaErrorInvalidConfiguration;
}

// Rotated-tier launches on st_rot, the others on st (the caller orders the two
// streams).
cudaError_t launch_quantize_tiles(const QuantParams& p, int dtype, cudaStream_t st, cudaStream_t st_rot) {
  if (dtype == GKV_BF16) return launch_tile_d<__nv_bfloat16>(p, st, st_rot);
  if (dtype == GKV_F16) return launch_tile_d<__half>(p, st, st_rot);
  return launch_tile_d<float>(p, st, st_rot);
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
