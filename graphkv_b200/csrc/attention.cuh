// Attention of queries over a compressed layer, reading the packed codes directly
// (the consumer of the compressed cache; the reference computes the same result as
// softmax(q k^T / sqrt(D)) v over the dequantized cache, core.py:800-820).
//
// One block of 128 threads per tile of 64 rows of one tier of one (batch, head)
// slice -- the dequantizer's tiles: retained rows, then standard, then cold.  The
// block decodes the tile's key and value rows into shared memory with the
// dequantizer's own decoders, so the rows it attends over are bit-identical to the
// dequantized cache's, and writes, per query, the tile's softmax partials: the
// largest logit m, the sum l of exp(logit - m) and o = sum exp(logit - m) v.  A
// second kernel merges the partials of a slice's tiles (rescaled to the overall
// largest logit) into the output, in two stages when a slice has many tiles.
// Only the summation order differs from the reference's fp32 matmul / softmax /
// matmul.
#pragma once

#include "dequantize.cuh"

namespace gkv {

constexpr int kAttnMaxQueries = 16;

struct AttnParams {
  DequantParams d;     // tiles, tiers and tensors of the layer (out_k / out_v unused)
  const float* q;      // [S, Q, D] fp32
  int Q;
  float inv_sqrt_d;    // 1 / sqrt(D)
  float* part;         // [S, tiles_slice, Q, D + 2]: m, l, o[D]
  float* part2;        // [S, merge groups, Q, D + 2]: the first merge stage's partials
  float* out;          // [S, Q, D] fp32
};

// Shared memory of a tile block: the decoded key and value tiles, the queries
// (Q x D fp32, 16-byte aligned size), then the tile's probabilities, 16 floats
// of reductions and D floats of partial value sums.
template <typename T, int D>
struct AGeom {
  using G = DGeom<T, D>;
  static constexpr size_t kTile = G::kTile;  // one decoded [64][D] tile
  static __host__ __device__ size_t q_bytes(int Q) { return ((size_t)Q * D * 4 + 15) & ~(size_t)15; }
  static __host__ __device__ size_t bytes(int Q) { return 2 * kTile + q_bytes(Q) + kDTile * 4 + 64 + D * 4; }
};

// Retained rows j0 .. j0 + rows of one tensor into a [64][D] tile (16-byte vectors).
template <typename T, int D>
__device__ __forceinline__ void load_retained_rows(const void* ret, int R, int s, int j0, int rows, uint8_t* tile) {
  using G = DGeom<T, D>;
  constexpr int CH = G::kRowBytes / 16;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(ret) + ((int64_t)s * R + j0) * G::kRowBytes;
  for (int i = threadIdx.x; i < rows * CH; i += kDThreads) {
    const int r = i / CH, c = i - r * CH;
    *reinterpret_cast<uint4*>(tile + r * G::kPitchB + c * 16) =
        *reinterpret_cast<const uint4*>(src + (int64_t)r * G::kRowBytes + c * 16);
  }
}

template <typename T, int D, bool VROT>
__global__ void __launch_bounds__(kDThreads, 6) attend_tile_kernel(const __grid_constant__ AttnParams a) {
  extern __shared__ __align__(128) uint8_t smem[];
  using G = DGeom<T, D>;
  using A = AGeom<T, D>;
  const DequantParams& p = a.d;
  uint8_t* tk = smem;
  uint8_t* tv = smem + A::kTile;
  float* qs = reinterpret_cast<float*>(smem + 2 * A::kTile);
  float* prob = reinterpret_cast<float*>(smem + 2 * A::kTile + A::q_bytes(a.Q));
  float* red = prob + kDTile;  // 16 floats of reductions, then D floats of partial sums
  const DTileRef tr = dtile_ref(p, blockIdx.x);
  const int s = tr.s;
  const int j0 = tr.k * kDTile;
  const int rows = min(kDTile, p.n_tier[tr.tier] - j0);
  // queries of this slice
  for (int i = threadIdx.x; i < a.Q * D; i += kDThreads) qs[i] = a.q[(int64_t)s * a.Q * D + i];
  // key and value rows of the tile
  if (tr.tier == 0) {
    load_retained_rows<T, D>(p.ret_k, p.n_tier[0], s, j0, rows, tk);
    load_retained_rows<T, D>(p.ret_v, p.n_tier[0], s, j0, rows, tv);
  } else {
    const TensorDesc& dk = p.t[tr.tier == 1 ? GKV_STD_K : GKV_COLD_K];
    const TensorDesc& dv = p.t[tr.tier == 1 ? GKV_STD_V : GKV_COLD_V];
    if (dk.sbits == 4) tok_decode<T, D, 4>(dk, s, j0, tk);
    else if (dk.sbits == 2) tok_decode<T, D, 2>(dk, s, j0, tk);
    else tok_decode<T, D, 8>(dk, s, j0, tk);
    constexpr int RUN = G::kRun;
    if (dv.rotation) {
      if constexpr (VROT) chan_decode_any<T, D, (RUN / 2 >= 32 && D / (RUN / 2) <= 4) ? RUN / 2 : RUN, true>(
          p, dv, s, j0, rows, tv);
    } else if (dv.gs < RUN) {
      if constexpr (RUN / 2 >= 32 && D / (RUN / 2) <= 4) chan_decode_any<T, D, RUN / 2, false>(p, dv, s, j0, rows, tv);
    } else {
      chan_decode_any<T, D, RUN, false>(p, dv, s, j0, rows, tv);
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = threadIdx.x >> 1, half = threadIdx.x & 1;  // two threads per tile row
  constexpr int HD = D / 2;
  float* part = a.part + ((int64_t)s * p.tiles_slice + (blockIdx.x - s * p.tiles_slice)) * a.Q * (D + 2);
  for (int qi = 0; qi < a.Q; ++qi) {
    const float* q = qs + qi * D;
    // logit of row r: q . k_r / sqrt(D)
    float dot = 0.f;
    if constexpr (sizeof(T) == 2) {  // 8 elements per 16-byte load
      using W = Word16<T>;
      const uint4* krow = reinterpret_cast<const uint4*>(tk + r * G::kPitchB + half * HD * 2);
      const float4* qh = reinterpret_cast<const float4*>(q + half * HD);
#pragma unroll 4
      for (int c8 = 0; c8 < HD / 8; ++c8) {
        const uint4 w = krow[c8];
        const float4 qa = qh[2 * c8], qb = qh[2 * c8 + 1];
        dot = __fmaf_rn(qa.x, W::lo(w.x), dot);
        dot = __fmaf_rn(qa.y, W::hi(w.x), dot);
        dot = __fmaf_rn(qa.z, W::lo(w.y), dot);
        dot = __fmaf_rn(qa.w, W::hi(w.y), dot);
        dot = __fmaf_rn(qb.x, W::lo(w.z), dot);
        dot = __fmaf_rn(qb.y, W::hi(w.z), dot);
        dot = __fmaf_rn(qb.z, W::lo(w.w), dot);
        dot = __fmaf_rn(qb.w, W::hi(w.w), dot);
      }
    } else {
      const T* krow = reinterpret_cast<const T*>(tk + r * G::kPitchB) + half * HD;
#pragma unroll 8
      for (int c = 0; c < HD; ++c) dot = __fmaf_rn(q[half * HD + c], Elem<T>::to_f32(krow[c]), dot);
    }
    dot += __shfl_xor_sync(kFull, dot, 1);
    const float logit = r < rows ? dot * a.inv_sqrt_d : -INFINITY;
    float m = logit;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float e = r < rows ? expf(logit - m) : 0.f;
    if (half == 0) prob[r] = e;
    float l = half == 0 ? e : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(kFull, l, o);
    __syncthreads();  // prob complete; red reads done
    if (lane == 0) red[4 + warp] = l;
    __syncthreads();
    // o[c] = sum_r prob[r] v_r[c]
    if constexpr (sizeof(T) == 2 && D == 128) {
      // thread: channels 2p, 2p + 1 over rows 32h .. 32h + 31 (p = tid % 64,
      // h = tid / 64); the two halves of the rows are added through shared memory
      using W = Word16<T>;
      const int pc = threadIdx.x & 63, h = threadIdx.x >> 6;
      float a0 = 0.f, a1 = 0.f;
      const int r0 = 32 * h, r1 = min(rows, r0 + 32);
#pragma unroll 4
      for (int rr = r0; rr < r1; ++rr) {
        const float pr = prob[rr];
        const uint32_t w = reinterpret_cast<const uint32_t*>(tv + rr * G::kPitchB)[pc];
        a0 = __fmaf_rn(pr, W::lo(w), a0);
        a1 = __fmaf_rn(pr, W::hi(w), a1);
      }
      float* oh = red + 16;  // D floats
      if (h == 1) {
        oh[2 * pc] = a0;
        oh[2 * pc + 1] = a1;
      }
      __syncthreads();
      if (h == 0) {
        part[qi * (D + 2) + 2 + 2 * pc] = a0 + oh[2 * pc];
        part[qi * (D + 2) + 3 + 2 * pc] = a1 + oh[2 * pc + 1];
      }
    } else {
      for (int c = threadIdx.x; c < D; c += kDThreads) {
        float acc = 0.f;
        for (int rr = 0; rr < rows; ++rr)
          acc = __fmaf_rn(prob[rr], Elem<T>::to_f32(reinterpret_cast<const T*>(tv + rr * G::kPitchB)[c]), acc);
        part[qi * (D + 2) + 2 + c] = acc;
      }
    }
    if (threadIdx.x == 0) {
      part[qi * (D + 2)] = m;
      part[qi * (D + 2) + 1] = red[4] + red[5] + red[6] + red[7];
    }
    __syncthreads();  // red / prob reused by the next query
  }
}

// Merge softmax partials (m, l, o[D]) in groups: one block of 256 threads per
// (slice, query, group of entries): the largest logit M over the group, each
// entry's weight exp(m_j - M) (kept in shared memory), L = sum of the weighted
// l_j and o = sum of the weighted o_j, with the entries split over the block's
// two halves (128 channels each).  FINAL (one group per slice): writes o / L;
// otherwise writes the group's own partial (M, L, o).  Partials are laid out
// [S][n][Q][D + 2].
constexpr int kCombineThreads = 256;
constexpr int kCombineSmemTiles = 8192;  // weights kept in shared memory up to this many entries
constexpr int kMergeGroup = 16;          // entries per block of the first merge stage

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(kFull, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < kCombineThreads / 32; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

template <bool FINAL>
__global__ void __launch_bounds__(kCombineThreads) attend_merge_kernel(const float* in, int n_in, int group, int Q,
                                                                         int D, float* out) {
  __shared__ float wts[kCombineSmemTiles];
  __shared__ float red[kCombineThreads / 32];
  __shared__ float half_o[2][128];
  const int ng = (n_in + group - 1) / group;
  const int sq = blockIdx.x / ng, g = blockIdx.x - sq * ng;  // (slice * Q + query, group)
  const int s = sq / Q, qi = sq - s * Q;
  const int j0 = g * group, n = min(n_in, j0 + group) - j0;
  const int64_t stride = (int64_t)Q * (D + 2);
  const float* part = in + ((int64_t)s * n_in + j0) * stride + (int64_t)qi * (D + 2);
  float m = -INFINITY;
  for (int j = threadIdx.x; j < n; j += kCombineThreads) m = fmaxf(m, part[j * stride]);
  const float M = block_reduce(m, red, true);
  float l = 0.f;
  for (int j = threadIdx.x; j < n; j += kCombineThreads) {
    const float w = expf(part[j * stride] - M);
    if (j < kCombineSmemTiles) wts[j] = w;
    l = __fmaf_rn(w, part[j * stride + 1], l);
  }
  const float L = block_reduce(l, red, false);  // its barriers also publish wts
  const int c = threadIdx.x & 127, h = threadIdx.x >> 7;
  float o = 0.f;
  if (c < D) {
#pragma unroll 4
    for (int j = h; j < n; j += 2) {
      const float w = j < kCombineSmemTiles ? wts[j] : expf(part[j * stride] - M);
      o = __fmaf_rn(w, part[j * stride + 2 + c], o);
    }
  }
  half_o[h][c] = o;
  __syncthreads();
  if (h == 0 && c < D) {
    const float sum = half_o[0][c] + half_o[1][c];
    if constexpr (FINAL) {
      out[(int64_t)sq * D + c] = sum / L;
    } else {
      float* dst = out + ((int64_t)s * ng + g) * stride + (int64_t)qi * (D + 2);
      if (c == 0) {
        dst[0] = M;
        dst[1] = L;
      }
      dst[2 + c] = sum;
    }
  }
}

// Entries of the first merge stage's output per slice (0: one stage).
__host__ __device__ inline int merge_groups(int tiles_slice) {
  return tiles_slice > 2 * kMergeGroup ? (tiles_slice + kMergeGroup - 1) / kMergeGroup : 0;
}

template <typename T, int D>
static cudaError_t launch_attention_t(const AttnParams& a, cudaStream_t st) {
  const size_t sm = AGeom<T, D>::bytes(a.Q);
  const bool vrot = (a.d.tiles[1] && a.d.t[GKV_STD_V].rotation) || (a.d.tiles[2] && a.d.t[GKV_COLD_V].rotation);
  auto kern = vrot ? attend_tile_kernel<T, D, true> : attend_tile_kernel<T, D, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)((int64_t)a.d.S * a.d.tiles_slice), kDThreads, sm, st>>>(a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const int n = a.d.tiles_slice, ng = merge_groups(n);
  if (ng > 0) {  // groups of kMergeGroup tiles, then their ng partials
    attend_merge_kernel<false><<<(unsigned)((int64_t)a.d.S * a.Q * ng), kCombineThreads, 0, st>>>(
        a.part, n, kMergeGroup, a.Q, D, a.part2);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    attend_merge_kernel<true><<<(unsigned)(a.d.S * a.Q), kCombineThreads, 0, st>>>(a.part2, ng, ng, a.Q, D, a.out);
  } else {
    attend_merge_kernel<true><<<(unsigned)(a.d.S * a.Q), kCombineThreads, 0, st>>>(a.part, n, n, a.Q, D, a.out);
  }
  return cudaGetLastError();
}

cudaError_t launch_attention(const AttnParams& a, int dtype, cudaStream_t st) {
  if (dtype == GKV_BF16) return a.d.D == 64 ? launch_attention_t<__nv_bfloat16, 64>(a, st)
                                            : launch_attention_t<__nv_bfloat16, 128>(a, st);
  if (dtype == GKV_F16) return a.d.D == 64 ? launch_attention_t<__half, 64>(a, st)
                                           : launch_attention_t<__half, 128>(a, st);
  return a.d.D == 64 ? launch_attention_t<float, 64>(a, st) : launch_attention_t<float, 128>(a, st);
}

}  // namespace gkv
