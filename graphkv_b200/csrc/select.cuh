// Tier selection (core.py:595-644, 685-719, 1034-1048) and outlier scores
// (core.py:1051-1054).
//
// One block of 1024 threads walks the T tokens.  Each top-k / bottom-k step is an
// MSB-first radix select over 32-bit order keys of the fp32 scores (4 passes of 8
// bits, histogram in shared memory with warp-aggregated atomics) that yields the
// k-th key; an ordered pass then marks every candidate beyond that key plus the
// lowest-position candidates equal to it.  A final ordered pass compacts the three
// ascending index lists.  A one-byte tier per token lives in the workspace.
#pragma once

#include "gkv_common.cuh"

namespace gkv {

namespace {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelSmemTokens = 40960;  // keys (4 B) + tier (1 B) per token fit in shared memory
enum : uint8_t { kCand = 0, kRet = 1, kCold = 2 };

struct SelectParams {
  const float* scores;
  const float* outlier;
  int T, sink, tail, keep_protect, keep_outlier, keep_cold;
  int n_ret, n_std, n_cold;
  uint8_t* tier;  // workspace (used when T exceeds kSelSmemTokens)
  int* idx_ret;
  int* idx_std;
  int* idx_cold;
};

// Monotone key: larger score -> larger key; NaN above +inf (torch.topk ranks NaN
// highest); -0.0 and +0.0 equal.
__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t b = __float_as_uint(f);
  if (f != f) b = 0x7FC00000u;
  if (f == 0.f) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct SelShared {
  uint32_t hist[256];
  uint32_t warp_cnt[3][kSelWarps];
  uint32_t warp_off[3][kSelWarps];
  uint32_t prefix, mask, remaining;
};

// Tokens handled by warp w in the ordered passes: one contiguous chunk per warp.
struct Chunk {
  int begin, end;
};
__device__ __forceinline__ Chunk warp_chunk(int T, int w) {
  const int per = ((T + kSelWarps - 1) / kSelWarps + 31) & ~31;
  const int b = min(T, w * per);
  return {b, min(T, b + per)};
}

// Exclusive scan of the per-warp counters (n of them) into warp_off; one barrier pair.
__device__ __forceinline__ void scan_warp_counts(SelShared& sh, int n) {
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp < n) {
    const uint32_t v = sh.warp_cnt[warp][lane];
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= o) inc += t;
    }
    sh.warp_off[warp][lane] = inc - v;
  }
  __syncthreads();
}

template <bool SMEM>
struct SelState {
  const uint32_t* keys;  // shared-memory keys (SMEM) of the importance scores
  uint8_t* tier;
};

template <bool SMEM>
__device__ __forceinline__ uint32_t key_at(const SelState<SMEM>& st, const float* src, int t) {
  if (SMEM && src == nullptr) return st.keys[t];
  return order_key(src[t]);
}

// Select `k` candidates (tier == kCand) with the largest (or smallest) keys and
// give them tier `mark`.  src == nullptr: the importance scores (cached keys).
template <bool SMEM>
__device__ void select_mark(const SelectParams& p, const SelState<SMEM>& st, const float* src, int k, bool largest,
                            uint8_t mark, SelShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) { sh.prefix = 0; sh.mask = 0; sh.remaining = (uint32_t)k; }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += kSelThreads) sh.hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = sh.prefix, mask = sh.mask;
    for (int base = 0; base < p.T; base += kSelThreads) {
      const int t = base + threadIdx.x;
      bool act = false;
      uint32_t digit = 0;
      if (t < p.T && st.tier[t] == kCand) {
        const uint32_t key = key_at<SMEM>(st, src, t);
        if ((key & mask) == prefix) {
          act = true;
          digit = (key >> shift) & 0xFFu;
        }
      }
      const uint32_t am = __ballot_sync(0xFFFFFFFFu, act);
      if (act) {
        const uint32_t peers = __match_any_sync(am, digit);
        if (lane == (__ffs(peers) - 1)) atomicAdd(&sh.hist[digit], __popc(peers));
      }
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns 8 bins in scan order (descending digits for `largest`)
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int bin = largest ? 255 - (lane * 8 + j) : lane * 8 + j;
        c[j] = sh.hist[bin];
        sum += c[j];
      }
      uint32_t inc = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += t;
      }
      const uint32_t rem = sh.remaining;
      const uint32_t before = inc - sum;
      const uint32_t hit = __ballot_sync(0xFFFFFFFFu, before < rem && inc >= rem);
      if (hit == 0) {
        // fewer candidates than requested: the count check at the end reports it
        if (lane == 0) { sh.remaining = rem; sh.prefix = prefix; sh.mask = mask | (0xFFu << shift); }
      } else if (lane == __ffs(hit) - 1) {
        uint32_t cum = before;
        int j = 0;
        for (; j < 8; ++j) {
          if (cum + c[j] >= rem) break;
          cum += c[j];
        }
        const int bin = largest ? 255 - (lane * 8 + j) : lane * 8 + j;
        sh.remaining = rem - cum;
        sh.prefix = prefix | ((uint32_t)bin << shift);
        sh.mask = mask | (0xFFu << shift);
      }
    }
    __syncthreads();
  }
  const uint32_t tau = sh.prefix;
  const uint32_t take_eq = sh.remaining;
  const Chunk ch = warp_chunk(p.T, warp);
  // pass 1: candidates equal to the k-th key, per warp chunk
  uint32_t cnt = 0;
  for (int b = ch.begin; b < ch.end; b += 32) {
    const int t = b + lane;
    const bool eq = t < ch.end && st.tier[t] == kCand && key_at<SMEM>(st, src, t) == tau;
    cnt += __popc(__ballot_sync(0xFFFFFFFFu, eq));
  }
  if (lane == 0) sh.warp_cnt[0][warp] = cnt;
  scan_warp_counts(sh, 1);
  // pass 2: mark keys beyond the k-th, and the first take_eq equal ones in token order
  uint32_t running = sh.warp_off[0][warp];
  for (int b = ch.begin; b < ch.end; b += 32) {
    const int t = b + lane;
    bool cand = false, beyond = false, eq = false;
    if (t < ch.end && st.tier[t] == kCand) {
      cand = true;
      const uint32_t key = key_at<SMEM>(st, src, t);
      beyond = largest ? key > tau : key < tau;
      eq = key == tau;
    }
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, eq);
    const uint32_t pos = running + __popc(bal & ((1u << lane) - 1u));
    if (cand && (beyond || (eq && pos < take_eq))) st.tier[t] = mark;
    running += __popc(bal);
  }
  __syncthreads();
}

template <bool SMEM>
__device__ void select_body(const SelectParams& p, SelState<SMEM> st, SelShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t = threadIdx.x; t < p.T; t += kSelThreads) {
    st.tier[t] = (t < p.sink || t >= p.T - p.tail) ? kRet : kCand;
    if (SMEM && p.scores) const_cast<uint32_t*>(st.keys)[t] = order_key(p.scores[t]);
  }
  __syncthreads();
  if (p.keep_protect > 0) select_mark<SMEM>(p, st, SMEM ? nullptr : p.scores, p.keep_protect, true, kRet, sh);
  if (p.keep_outlier > 0) select_mark<SMEM>(p, st, p.outlier, p.keep_outlier, true, kRet, sh);
  if (p.keep_cold > 0) select_mark<SMEM>(p, st, SMEM ? nullptr : p.scores, p.keep_cold, false, kCold, sh);
  // ordered compaction of the three lists
  const Chunk ch = warp_chunk(p.T, warp);
  uint32_t n[3] = {0, 0, 0};
  for (int b = ch.begin; b < ch.end; b += 32) {
    const int t = b + lane;
    const uint8_t c = t < ch.end ? st.tier[t] : 0xFF;
    n[0] += __popc(__ballot_sync(0xFFFFFFFFu, c == kRet));
    n[1] += __popc(__ballot_sync(0xFFFFFFFFu, c == kCand));
    n[2] += __popc(__ballot_sync(0xFFFFFFFFu, c == kCold));
  }
  if (lane == 0) {
    sh.warp_cnt[0][warp] = n[0];
    sh.warp_cnt[1][warp] = n[1];
    sh.warp_cnt[2][warp] = n[2];
  }
  scan_warp_counts(sh, 3);
  uint32_t off[3] = {sh.warp_off[0][warp], sh.warp_off[1][warp], sh.warp_off[2][warp]};
  int* const out[3] = {p.idx_ret, p.idx_std, p.idx_cold};
  const uint32_t lim[3] = {(uint32_t)p.n_ret, (uint32_t)p.n_std, (uint32_t)p.n_cold};
  const uint8_t code[3] = {kRet, kCand, kCold};
  for (int b = ch.begin; b < ch.end; b += 32) {
    const int t = b + lane;
    const uint8_t c = t < ch.end ? st.tier[t] : 0xFF;
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const uint32_t bal = __ballot_sync(0xFFFFFFFFu, c == code[q]);
      const uint32_t pos = off[q] + __popc(bal & ((1u << lane) - 1u));
      if (c == code[q] && pos < lim[q]) out[q][pos] = t;
      off[q] += __popc(bal);
    }
  }
  if (threadIdx.x == 0) {
    const uint32_t tot[3] = {sh.warp_off[0][31] + sh.warp_cnt[0][31], sh.warp_off[1][31] + sh.warp_cnt[1][31],
                             sh.warp_off[2][31] + sh.warp_cnt[2][31]};
    if (tot[0] != lim[0] || tot[1] != lim[1] || tot[2] != lim[2]) raise_error(kErrSelectCount);
  }
}

__global__ void __launch_bounds__(kSelThreads) select_kernel(const SelectParams p) {
  __shared__ SelShared sh;
  extern __shared__ __align__(16) uint8_t sel_smem[];
  if (p.T <= kSelSmemTokens) {
    SelState<true> st{reinterpret_cast<const uint32_t*>(sel_smem), sel_smem + 4 * (size_t)kSelSmemTokens};
    select_body<true>(p, st, sh);
  } else {
    SelState<false> st{nullptr, p.tier};
    select_body<false>(p, st, sh);
  }
}

// mean(K^2) + mean(V^2) per token: warp per token, fp64 accumulation
template <typename E>
__global__ void outlier_kernel(const gkv_layer_in L, int B, int T, int D, float* out) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (t >= T) return;
  double acc[2] = {0.0, 0.0};
  for (int which = 0; which < 2; ++which) {
    const E* base = reinterpret_cast<const E*>(which ? L.v : L.k);
    const int64_t* st = which ? L.v_stride : L.k_stride;
    double a = 0.0;
    for (int b = 0; b < B; ++b)
      for (int h = 0; h < L.heads; ++h) {
        const E* row = base + b * st[0] + h * st[1] + (int64_t)t * st[2];
        for (int c = lane; c < D; c += 32) {
          const double x = (double)Elem<E>::to_f32(row[c]);
          a += x * x;
        }
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    acc[which] = a;
  }
  if (lane == 0) {
    const double n = (double)B * L.heads * D;
    out[t] = __fadd_rn((float)(acc[0] / n), (float)(acc[1] / n));
  }
}

}  // namespace

cudaError_t launch_select(const float* scores, const float* outlier, const gkv_select_policy& pol, int* idx_ret,
                          int* idx_std, int* idx_cold, uint8_t* tier, cudaStream_t st) {
  SelectParams p;
  p.scores = scores;
  p.outlier = outlier;
  p.T = pol.seq_len;
  p.sink = pol.sink;
  p.tail = pol.tail;
  p.keep_protect = pol.keep_protect;
  p.keep_outlier = pol.keep_outlier;
  p.keep_cold = pol.keep_cold;
  p.n_ret = pol.n_retained;
  p.n_std = pol.n_standard;
  p.n_cold = pol.n_cold;
  p.tier = tier;
  p.idx_ret = idx_ret;
  p.idx_std = idx_std;
  p.idx_cold = idx_cold;
  const size_t sm = pol.seq_len <= kSelSmemTokens ? (size_t)kSelSmemTokens * 5 : 0;
  cudaError_t e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  select_kernel<<<1, kSelThreads, sm, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_outlier(const gkv_layer_in& L, int B, int T, int D, int dtype, float* out, cudaStream_t st) {
  const unsigned blocks = (unsigned)ceil_div(T, 8);
  if (dtype == GKV_BF16) outlier_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(L, B, T, D, out);
  else if (dtype == GKV_F16) outlier_kernel<__half><<<blocks, 256, 0, st>>>(L, B, T, D, out);
  else outlier_kernel<float><<<blocks, 256, 0, st>>>(L, B, T, D, out);
  return cudaGetLastError();
}

}  // namespace gkv
