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
enum : uint8_t { kCand = 0, kRet = 1, kCold = 2 };

struct SelectParams {
  const float* scores;
  const float* outlier;
  int T, sink, tail, keep_protect, keep_outlier, keep_cold;
  int n_ret, n_std, n_cold;
  uint8_t* tier;
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
  uint32_t warp_tot[kSelWarps];
  uint32_t scan[kSelWarps];
  uint32_t prefix, mask, remaining;
};

// exclusive block scan of one flag per thread; returns the prefix, total in *total
__device__ __forceinline__ uint32_t block_scan_flag(bool flag, SelShared& sh, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t bal = __ballot_sync(0xFFFFFFFFu, flag);
  const uint32_t in_warp = __popc(bal & ((1u << lane) - 1u));
  if (lane == 0) sh.warp_tot[warp] = __popc(bal);
  __syncthreads();
  if (warp == 0) {
    const uint32_t v = sh.warp_tot[lane];
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= o) inc += t;
    }
    sh.scan[lane] = inc - v;
    __syncwarp();
    if (lane == 31) sh.warp_tot[0] = inc;  // block total (slot 0 was read above)
  }
  __syncthreads();
  const uint32_t r = sh.scan[warp] + in_warp;
  *total = sh.warp_tot[0];
  __syncthreads();
  return r;
}

// Select `k` candidates (tier == kCand) with the largest (or smallest) keys of
// `src` and give them tier `mark`.
__device__ void select_mark(const SelectParams& p, const float* src, int k, bool largest, uint8_t mark,
                            SelShared& sh) {
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
      if (t < p.T && p.tier[t] == kCand) {
        const uint32_t key = order_key(src[t]);
        if ((key & mask) == prefix) {
          act = true;
          digit = (key >> shift) & 0xFFu;
        }
      }
      const uint32_t am = __ballot_sync(0xFFFFFFFFu, act);
      if (act) {
        const uint32_t peers = __match_any_sync(am, digit);
        if ((threadIdx.x & 31) == (__ffs(peers) - 1)) atomicAdd(&sh.hist[digit], __popc(peers));
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t rem = sh.remaining;
      uint32_t cum = 0;
      int d = 0;
      for (int step = 0; step < 256; ++step) {
        d = largest ? 255 - step : step;
        const uint32_t c = sh.hist[d];
        if (cum + c >= rem) break;
        cum += c;
      }
      sh.remaining = rem - cum;
      sh.prefix = prefix | ((uint32_t)d << shift);
      sh.mask = mask | (0xFFu << shift);
    }
    __syncthreads();
  }
  const uint32_t tau = sh.prefix;
  const uint32_t take_eq = sh.remaining;
  uint32_t running = 0;
  for (int base = 0; base < p.T; base += kSelThreads) {
    const int t = base + threadIdx.x;
    bool cand = false, beyond = false, eq = false;
    if (t < p.T && p.tier[t] == kCand) {
      cand = true;
      const uint32_t key = order_key(src[t]);
      beyond = largest ? key > tau : key < tau;
      eq = key == tau;
    }
    uint32_t total;
    const uint32_t pos = block_scan_flag(eq, sh, &total);
    if (cand && (beyond || (eq && running + pos < take_eq))) p.tier[t] = mark;
    running += total;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kSelThreads) select_kernel(const SelectParams p) {
  __shared__ SelShared sh;
  for (int t = threadIdx.x; t < p.T; t += kSelThreads)
    p.tier[t] = (t < p.sink || t >= p.T - p.tail) ? kRet : kCand;
  __syncthreads();
  if (p.keep_protect > 0) select_mark(p, p.scores, p.keep_protect, true, kRet, sh);
  if (p.keep_outlier > 0) select_mark(p, p.outlier, p.keep_outlier, true, kRet, sh);
  if (p.keep_cold > 0) select_mark(p, p.scores, p.keep_cold, false, kCold, sh);
  uint32_t nr = 0, ns = 0, nc = 0;
  for (int base = 0; base < p.T; base += kSelThreads) {
    const int t = base + threadIdx.x;
    const uint8_t c = t < p.T ? p.tier[t] : 0xFF;
    uint32_t tr, ts, tc;
    const uint32_t pr = block_scan_flag(c == kRet, sh, &tr);
    const uint32_t ps = block_scan_flag(c == kCand, sh, &ts);
    const uint32_t pc = block_scan_flag(c == kCold, sh, &tc);
    if (c == kRet && nr + pr < (uint32_t)p.n_ret) p.idx_ret[nr + pr] = t;
    if (c == kCand && ns + ps < (uint32_t)p.n_std) p.idx_std[ns + ps] = t;
    if (c == kCold && nc + pc < (uint32_t)p.n_cold) p.idx_cold[nc + pc] = t;
    nr += tr;
    ns += ts;
    nc += tc;
  }
  if (threadIdx.x == 0 && (nr != (uint32_t)p.n_ret || ns != (uint32_t)p.n_std || nc != (uint32_t)p.n_cold))
    raise_error(kErrSelectCount);
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
  select_kernel<<<1, kSelThreads, 0, st>>>(p);
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
