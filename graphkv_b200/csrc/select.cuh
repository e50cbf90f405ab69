// Tier selection (core.py:595-644, 685-719, 1034-1048) and outlier scores
// (core.py:1051-1054).
//
// One block of 1024 threads walks the T tokens.  Each top-k / bottom-k step is an
// MSB-first radix select over 32-bit order keys of the fp32 scores (4 passes of 8
// bits, histogram in shared memory with warp-aggregated atomics) that yields the
// k-th key.  When every candidate equal to that key is taken, the set is unique
// and an ordered pass marks it.  Otherwise (a tie straddles the boundary) the
// choice is the one torch.topk makes on the CPU, which follows the order libstdc++
// visits its queue of candidates: select_exact restates std::partial_sort's heap
// select (k * 64 <= n) and std::nth_element's introselect on the device.  A final
// ordered pass compacts the three ascending index lists.  Workspace: one tier byte
// per token, then the candidate queue and the two partition stop tables (int32).
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
  int* queue;     // workspace [T]: candidate queue of the exact tie path
  int* stop_l;    // workspace [T]: left stops of a partition, by rank
  int* stop_r;    // workspace [T]: right stops of a partition, by rank
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
  // exact tie path
  int first, last, depth, done;
  uint32_t pivot;
  int pairs;
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

// ---------------------------------------------------------------------------
// Exact tie path: the selection torch.topk makes on the CPU.
//
// ATen's CPU topk (TopKImpl.h, topk_impl_loop) fills a queue of (value,
// position) pairs in position order and runs std::partial_sort when
// k * 64 <= n, else std::nth_element, with the comparator "x > y" (largest) or
// "x < y" (smallest) on the values; the first k queue slots are the result.
// Which of several equal values lands there follows the libstdc++ algorithms
// (GCC bits/stl_heap.h, bits/stl_algo.h), restated here over order keys:
//  - heap select: heapify the first k slots, then each later element that
//    compares before the heap top replaces it (__adjust_heap + __push_heap);
//    serial in one thread, the scan for replacement candidates warp-parallel
//    (an element that does not beat the top cannot beat a later top);
//  - introselect: median-of-three pivot moved to `first`, unguarded Hoare
//    partition, continue on the side holding nth; heap select when the depth
//    limit 2*floor(log2 n) runs out; insertion sort of the last <= 3 slots.
//    The partition is computed in parallel: its m-th swap exchanges the m-th
//    left stop (a slot whose key does not compare before the pivot, counted
//    from the left) with the m-th right stop (a slot the pivot does not compare
//    before, counted from the right) while the left one lies left of the right
//    one.  The number of swaps M is the maximum over cut positions x of
//    min(#left stops left of x, #right stops at or right of x), and the split
//    point is the (M+1)-th left stop or, when the scanners meet on a swapped
//    slot, the M-th right stop.
// ---------------------------------------------------------------------------

template <bool SMEM>
struct KeyOf {
  const SelState<SMEM>& st;
  const float* src;
  __device__ __forceinline__ uint32_t operator()(int pos) const { return key_at<SMEM>(st, src, pos); }
};

struct Before {
  bool largest;
  __device__ __forceinline__ bool operator()(uint32_t a, uint32_t b) const { return largest ? a > b : a < b; }
};

// __adjust_heap followed by __push_heap on the heap q[first, first + len).
template <class Key>
__device__ void adjust_heap(int* q, int first, int hole, int len, int item, uint32_t item_key, const Key& key,
                            Before before) {
  const int top = hole;
  int child = hole;
  while (child < (len - 1) / 2) {
    child = 2 * (child + 1);
    if (before(key(q[first + child]), key(q[first + child - 1]))) --child;
    q[first + hole] = q[first + child];
    hole = child;
  }
  if ((len & 1) == 0 && child == (len - 2) / 2) {
    child = 2 * (child + 1);
    q[first + hole] = q[first + child - 1];
    hole = child - 1;
  }
  int parent = (hole - 1) / 2;
  while (hole > top && before(key(q[first + parent]), item_key)) {
    q[first + hole] = q[first + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  q[first + hole] = item;
}

template <class Key>
__device__ void make_heap(int* q, int first, int len, const Key& key, Before before) {
  if (len < 2) return;
  for (int parent = (len - 2) / 2;; --parent) {
    const int item = q[first + parent];
    adjust_heap(q, first, parent, len, item, key(item), key, before);
    if (parent == 0) break;
  }
}

// __heap_select(first, middle, last), one thread.
template <class Key>
__device__ void heap_select_serial(int* q, int first, int middle, int last, const Key& key, Before before) {
  const int len = middle - first;
  make_heap(q, first, len, key, before);
  uint32_t top = key(q[first]);
  for (int i = middle; i < last; ++i) {
    const int item = q[i];
    const uint32_t k = key(item);
    if (before(k, top)) {
      q[i] = q[first];
      adjust_heap(q, first, 0, len, item, k, key, before);
      top = key(q[first]);
    }
  }
}

// __heap_select(0, k, n) by warp 0: lanes test 32 slots at a time against the
// heap top; lane 0 replays the replacements in slot order.
template <class Key>
__device__ void heap_select_warp(int* q, int k, int n, const Key& key, Before before) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) make_heap(q, 0, k, key, before);
  __syncwarp();
  uint32_t top = __shfl_sync(0xFFFFFFFFu, lane == 0 ? key(q[0]) : 0u, 0);
  for (int base = k; base < n; base += 32) {
    const int i = base + lane;
    const int item = i < n ? q[i] : 0;
    const uint32_t ki = i < n ? key(item) : 0u;
    uint32_t hits = __ballot_sync(0xFFFFFFFFu, i < n && before(ki, top));
    while (hits) {
      const int l = __ffs(hits) - 1;
      hits &= hits - 1;
      const uint32_t kl = __shfl_sync(0xFFFFFFFFu, ki, l);
      const int il = __shfl_sync(0xFFFFFFFFu, item, l);
      if (before(kl, top)) {
        uint32_t nt = 0;
        if (lane == 0) {
          q[base + l] = q[0];
          adjust_heap(q, 0, 0, k, il, kl, key, before);
          nt = key(q[0]);
        }
        __syncwarp();
        top = __shfl_sync(0xFFFFFFFFu, nt, 0);
      }
    }
  }
  __syncwarp();
}

// __insertion_sort(first, last), one thread.
template <class Key>
__device__ void insertion_sort_serial(int* q, int first, int last, const Key& key, Before before) {
  for (int i = first + 1; i < last; ++i) {
    const int item = q[i];
    const uint32_t k = key(item);
    if (before(k, key(q[first]))) {
      for (int j = i; j > first; --j) q[j] = q[j - 1];
      q[first] = item;
    } else {
      int j = i;
      while (before(k, key(q[j - 1]))) {
        q[j] = q[j - 1];
        --j;
      }
      q[j] = item;
    }
  }
}

// Contiguous piece of [lo, hi) for warp w (multiples of 32 slots).
__device__ __forceinline__ Chunk range_chunk(int lo, int hi, int w) {
  const int len = hi - lo;
  const int per = ((len + kSelWarps - 1) / kSelWarps + 31) & ~31;
  const int b = min(hi, lo + w * per);
  return {b, min(hi, b + per)};
}

// Mark the k candidates torch.topk would choose.  The candidates are compacted
// into the queue in position order first.
template <bool SMEM>
__device__ void select_exact(const SelectParams& p, const SelState<SMEM>& st, const float* src, int k, bool largest,
                             uint8_t mark, SelShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int* const q = p.queue;
  const KeyOf<SMEM> key{st, src};
  const Before before{largest};
  // queue of candidates in position order
  const Chunk ch = warp_chunk(p.T, warp);
  uint32_t cnt = 0;
  for (int b = ch.begin; b < ch.end; b += 32) {
    const int t = b + lane;
    cnt += __popc(__ballot_sync(0xFFFFFFFFu, t < ch.end && st.tier[t] == kCand));
  }
  if (lane == 0) sh.warp_cnt[0][warp] = cnt;
  scan_warp_counts(sh, 1);
  uint32_t off = sh.warp_off[0][warp];
  for (int b = ch.begin; b < ch.end; b += 32) {
    const int t = b + lane;
    const bool c = t < ch.end && st.tier[t] == kCand;
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, c);
    if (c) q[off + __popc(bal & ((1u << lane) - 1u))] = t;
    off += __popc(bal);
  }
  const int n = (int)(sh.warp_off[0][kSelWarps - 1] + sh.warp_cnt[0][kSelWarps - 1]);
  __syncthreads();
  if (k > n) k = n;  // the count check reports the shortfall
  if (k <= 0) return;
  if ((int64_t)k * 64 <= n) {
    if (warp == 0) heap_select_warp(q, k, n, key, before);
  } else {
    const int nth = k - 1;
    if (threadIdx.x == 0) {
      sh.first = 0;
      sh.last = n;
      sh.depth = 2 * (31 - __clz(max(n, 1)));
      sh.done = 0;
    }
    __syncthreads();
    while (true) {
      const int first = sh.first, last = sh.last, done = sh.done, depth = sh.depth;
      __syncthreads();  // every thread has read the loop state before thread 0 updates it
      if (done || last - first <= 3) break;
      if (depth == 0) {
        if (threadIdx.x == 0) {
          heap_select_serial(q, first, nth + 1, last, key, before);
          const int t = q[first];
          q[first] = q[nth];
          q[nth] = t;
          sh.done = 2;
        }
        break;
      }
      if (threadIdx.x == 0) {
        sh.depth = depth - 1;
        const int a = first + 1, b = first + (last - first) / 2, c = last - 1;
        const uint32_t ka = key(q[a]), kb = key(q[b]), kc = key(q[c]);
        int m;
        if (before(ka, kb)) m = before(kb, kc) ? b : (before(ka, kc) ? c : a);
        else if (before(ka, kc)) m = a;
        else if (before(kb, kc)) m = c;
        else m = b;
        const int t = q[first];
        q[first] = q[m];
        q[m] = t;
        sh.pivot = key(q[first]);
        sh.pairs = 0;
      }
      __syncthreads();
      const uint32_t piv = sh.pivot;
      const int lo = first + 1, hi = last;
      const Chunk rc = range_chunk(lo, hi, warp);
      // pass 1: left / right stops per warp piece
      uint32_t nl = 0, nr = 0;
      for (int b = rc.begin; b < rc.end; b += 32) {
        const int i = b + lane;
        bool ls = false, rs = false;
        if (i < rc.end) {
          const uint32_t kk = key(q[i]);
          ls = !before(kk, piv);
          rs = !before(piv, kk);
        }
        nl += __popc(__ballot_sync(0xFFFFFFFFu, ls));
        nr += __popc(__ballot_sync(0xFFFFFFFFu, rs));
      }
      if (lane == 0) {
        sh.warp_cnt[0][warp] = nl;
        sh.warp_cnt[1][warp] = nr;
      }
      scan_warp_counts(sh, 2);
      const int total_l = (int)(sh.warp_off[0][kSelWarps - 1] + sh.warp_cnt[0][kSelWarps - 1]);
      const int total_r = (int)(sh.warp_off[1][kSelWarps - 1] + sh.warp_cnt[1][kSelWarps - 1]);
      // pass 2: ranks, stop tables and the swap count
      uint32_t left_before = sh.warp_off[0][warp], right_before = sh.warp_off[1][warp];
      int best = 0;
      for (int b = rc.begin; b < rc.end; b += 32) {
        const int i = b + lane;
        bool ls = false, rs = false;
        if (i < rc.end) {
          const uint32_t kk = key(q[i]);
          ls = !before(kk, piv);
          rs = !before(piv, kk);
        }
        const uint32_t bl = __ballot_sync(0xFFFFFFFFu, ls), br = __ballot_sync(0xFFFFFFFFu, rs);
        const uint32_t below = (1u << lane) - 1u;
        const int lrank = (int)(left_before + __popc(bl & below));     // left stops in [lo, i)
        const int rbefore = (int)(right_before + __popc(br & below));  // right stops in [lo, i)
        if (ls) p.stop_l[lrank] = i;
        if (rs) p.stop_r[total_r - 1 - rbefore] = i;
        if (i < rc.end) best = max(best, min(lrank, total_r - rbefore));  // cut just before slot i
        left_before += __popc(bl);
        right_before += __popc(br);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
      if (lane == 0 && best > 0) atomicMax(&sh.pairs, best);
      __syncthreads();
      const int pairs = sh.pairs;
      // pass 3: the swaps (disjoint slot pairs)
      for (int m = threadIdx.x; m < pairs; m += kSelThreads) {
        const int i = p.stop_l[m], j = p.stop_r[m];
        const int t = q[i];
        q[i] = q[j];
        q[j] = t;
      }
      if (threadIdx.x == 0) {
        int cut = -1;
        if (pairs >= 1 && !(pairs < total_l && p.stop_l[pairs] < p.stop_r[pairs - 1])) cut = p.stop_r[pairs - 1];
        else if (pairs < total_l) cut = p.stop_l[pairs];
        if (cut < 0) {  // unreachable: the median of three guards the left scan
          raise_error(kErrSelectCount);
          sh.done = 1;
        } else if (cut <= nth) {
          sh.first = cut;
        } else {
          sh.last = cut;
        }
      }
      __syncthreads();
    }
    __syncthreads();
    if (threadIdx.x == 0 && sh.done == 0) insertion_sort_serial(q, sh.first, sh.last, key, before);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < k; i += kSelThreads) st.tier[q[i]] = mark;
  __syncthreads();
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
  const uint32_t n_eq = sh.warp_off[0][kSelWarps - 1] + sh.warp_cnt[0][kSelWarps - 1];
  if (take_eq < n_eq) {  // a tie straddles the boundary
    select_exact<SMEM>(p, st, src, k, largest, mark, sh);
    return;
  }
  // pass 2: mark keys beyond the k-th and every key equal to it
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

// Workspace of the select kernel: tier bytes [T], then queue, left and right stop
// tables (int32 [T] each), every region 256-byte aligned.
constexpr size_t select_region(int T) { return ((size_t)T * 4 + 255) & ~(size_t)255; }
constexpr size_t select_workspace(int T) { return (((size_t)T + 255) & ~(size_t)255) + 3 * select_region(T); }

cudaError_t launch_select(const float* scores, const float* outlier, const gkv_select_policy& pol, int* idx_ret,
                          int* idx_std, int* idx_cold, uint8_t* workspace, cudaStream_t st) {
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
  const int T = pol.seq_len;
  uint8_t* w = workspace;
  p.tier = w;
  w += ((size_t)T + 255) & ~(size_t)255;
  p.queue = reinterpret_cast<int*>(w);
  p.stop_l = reinterpret_cast<int*>(w + select_region(T));
  p.stop_r = reinterpret_cast<int*>(w + 2 * select_region(T));
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
