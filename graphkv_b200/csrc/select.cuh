// Tier selection (core.py:595-644, 685-719, 1034-1048) and outlier scores
// (core.py:1051-1054).
//
// A cluster of 8 blocks of 1024 threads walks the T tokens: block r owns one
// contiguous range of them, with their order keys and tier bytes in its shared
// memory.  Each top-k / bottom-k step is an MSB-first radix select over 32-bit
// order keys of the fp32 scores (digits of 11, 11 and 10 bits): every block counts
// the digit of its own candidates into a histogram in its shared memory (warp-
// aggregated atomics), and after a cluster barrier every block reads the eight
// histograms through distributed shared memory and finds the same bin of the k-th
// key.  When every candidate equal to that key is taken, the set is unique: "at or
// beyond the k-th key", marked by the next sweep.  Otherwise (a tie straddles the
// boundary) the choice is the one torch.topk makes on the CPU, which follows the
// order libstdc++ visits its queue of candidates: select_exact restates
// std::partial_sort's heap select (k * 64 <= n) and std::nth_element's introselect,
// run by block 0 over the tier bytes in global memory.  A final ordered pass
// compacts the three ascending index lists, each block at the offsets of the
// blocks before it.  Workspace: one tier byte per token, then the candidate queue
// (positions and keys) and the partition stop tables (int32).
#pragma once

#include <algorithm>

#include <cooperative_groups.h>

#include "gkv_common.cuh"

namespace gkv {

namespace {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelCluster = 8;         // blocks of the selection cluster
constexpr int kSelSmemTokens = 40960;  // tokens per block whose keys (4 B) and tier (1 B) fit in shared memory
constexpr size_t kSelSmemLimit = 227 * 1024;  // shared memory of one block (static + dynamic)
constexpr size_t kSelExactSmem = 48 * 1024;   // least dynamic shared memory (the exact path's scratch)
constexpr int kSelWindow = 4096;              // heap select: queue entries filtered per window
enum : uint8_t { kCand = 0, kRet = 1, kCold = 2 };

struct SelectParams {
  const float* scores;
  const float* outlier;
  int T, sink, tail, keep_protect, keep_outlier, keep_cold;
  int n_ret, n_std, n_cold;
  uint8_t* tier;  // workspace: tier bytes (blocks of more than kSelSmemTokens tokens, exact path)
  int* queue;       // workspace [T]: candidate positions of the exact tie path
  uint32_t* qkey;   // workspace [T]: their order keys
  int* stops;       // workspace [T + 1]: stop tables of a partition (or the heap nodes)
  int* idx_ret;
  int* idx_std;
  int* idx_cold;
  int smem_bytes;      // dynamic shared memory of each block (the exact path's scratch in block 0)
};

// Monotone key: larger score -> larger key; NaN above +inf (torch.topk ranks NaN
// highest); -0.0 and +0.0 equal.
__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t b = __float_as_uint(f);
  if (f != f) b = 0x7FC00000u;
  if (f == 0.f) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kBins = 2048;  // 11-bit digits

struct SelShared {
  uint32_t hist[3][kBins];  // 0, 1: alternate digit passes, so a block clears one while peers read the
                            // other; 2: the first selection's first-digit counts, kept for the cold tier
  uint32_t saved_bin;       // the first selection's first-digit bin
  uint32_t warp_cnt[3][kSelWarps];
  uint32_t warp_off[3][kSelWarps];
  uint32_t wsum[kSelWarps];
  uint32_t list_tot[3];   // this block's count of each list
  uint32_t list_off[3];   // counts of the blocks before it
  uint32_t list_all[3];   // whole cluster
  uint32_t pick_bin, pick_rem, pick_cnt;
  int found;
  // exact tie path
  int first, last, depth, done;
  uint32_t pivot;
  int pairs;
};

namespace cg = cooperative_groups;
__device__ __forceinline__ void cluster_sync() { cg::this_cluster().sync(); }
// The same shared-memory object in block r of the cluster.
template <class U>
__device__ __forceinline__ U* peer(U* p, int r) {
  return cg::this_cluster().map_shared_rank(p, r);
}
// 32-bit word at the same shared-memory address in block r, read through the
// cluster's shared window.
__device__ __forceinline__ uint32_t ld_peer(const uint32_t* p, int r) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(p), ra, v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(r));
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(ra) : "memory");
  return v;
}

// Tokens handled by warp w in the sweeps of [lo, hi): one contiguous chunk per
// warp, a multiple of 128 tokens (four 32-token slices per step).
struct Chunk {
  int begin, end;
};
__device__ __forceinline__ Chunk warp_chunk(int lo, int hi, int w) {
  const int per = ((hi - lo + kSelWarps - 1) / kSelWarps + 127) & ~127;
  const int b = min(hi, lo + w * per);
  return {b, min(hi, b + per)};
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

// Tokens [base, end) of this block.  SMEM: keys of the importance scores and
// tier bytes in shared memory, indexed from base; otherwise tier points at the
// workspace byte of token base and keys are read from the scores.
template <bool SMEM>
struct SelState {
  uint32_t* keys;
  uint8_t* tier;
  int base, end;
};

template <bool SMEM>
__device__ __forceinline__ uint32_t key_at(const SelState<SMEM>& st, const float* src, int t) {
  if (SMEM && src == nullptr) return st.keys[t - st.base];
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
//    compares before the heap top replaces it (__adjust_heap + __push_heap,
//    restated as one top-down pass); the replacements are serial in one thread,
//    the scan for them warp-parallel (an element that does not beat the top
//    cannot beat a later top);
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

struct Before {
  bool largest;
  __device__ __forceinline__ bool operator()(uint32_t a, uint32_t b) const { return largest ? a > b : a < b; }
};
// The same order with the direction fixed at compile time (the heap select's
// serial sifts).
template <bool LARGEST>
struct BeforeC {
  __device__ __forceinline__ bool operator()(uint32_t a, uint32_t b) const { return LARGEST ? a > b : a < b; }
};

// The candidate queue of the exact path: positions q[i] and their order keys
// qk[i], moved together (so no pass gathers keys through positions).
struct Queue {
  int* q;
  uint32_t* qk;
  __device__ __forceinline__ void swap(int i, int j) const {
    const int t = q[i];
    q[i] = q[j];
    q[j] = t;
    const uint32_t u = qk[i];
    qk[i] = qk[j];
    qk[j] = u;
  }
};

// Contiguous piece of [lo, hi) for warp w (multiples of 128 slots).
__device__ __forceinline__ Chunk range_chunk(int lo, int hi, int w) {
  const int len = hi - lo;
  const int per = ((len + kSelWarps - 1) / kSelWarps + 127) & ~127;
  const int b = min(hi, lo + w * per);
  return {b, min(hi, b + per)};
}

// Heap nodes {key, position}; node i of a heap lives at nd[i + 1], so the two
// children 2i + 1, 2i + 2 of a node share one 16-byte word and its four
// grandchildren 4i + 3 .. 4i + 6 two more.  Entries beyond the heap's length
// (up to index len + 3) are read but never used.
//
// sift_down(h, x): libstdc++'s __adjust_heap(first, h, len, x) followed by
// __push_heap, restated top-down.  __adjust_heap moves the hole from h to a leaf
// along the path of chosen children (the right child unless comp(right, left))
// and __push_heap moves x back up while comp(parent, x).  Along that path no
// parent compares before its child (heap order), so the nodes that compare
// before x form a tail of the path, which __push_heap restores to where they
// were: walking down and stopping at the first chosen child that compares
// before x leaves the same heap.  The loads of the next level's pair of
// children are issued one level ahead.  Returns the key at the root afterwards.
__host__ __device__ constexpr size_t heap_node_bytes(int cap) { return 8 * ((size_t)cap + 8); }

template <class Cmp>
__device__ __forceinline__ uint32_t sift_down(uint2* nd, int h, int len, uint2 x, Cmp before) {
  // A uniform number of levels (the depth below h), with the moves predicated
  // and the loads unconditional (node pair 0 stands in past the heap's end), so
  // no branch waits on a loaded key; the next pair of children is loaded one
  // level ahead.
  const int h0 = h;
  uint32_t root = x.x;
  const int levels = (31 - __clz(len)) - (31 - __clz(h0 + 1));
  bool go = true;
  int l = 2 * h + 1;
  uint4 c = *reinterpret_cast<const uint4*>(nd + (l < len ? l + 1 : 0));
  for (int it = 0; it < levels; ++it) {
    const int gl = 2 * l + 1;  // first grandchild
    const bool gok = gl < len;
    const uint4 g0 = *reinterpret_cast<const uint4*>(nd + (gok ? gl + 1 : 0));
    const uint4 g1 = *reinterpret_cast<const uint4*>(nd + (gok ? gl + 3 : 0));
    const bool has = go && l < len;
    const bool right = l + 1 < len && !before(c.z, c.x);
    const uint2 ch = right ? make_uint2(c.z, c.w) : make_uint2(c.x, c.y);
    go = has && !before(ch.x, x.x);
    if (go) nd[h + 1] = ch;
    root = (go && h == h0) ? ch.x : root;
    h = go ? (right ? l + 1 : l) : h;
    l = go ? 2 * h + 1 : l;
    c = right ? g1 : g0;
  }
  nd[h + 1] = x;
  return root;
}

// std::make_heap over nodes 0 .. len - 1 by one warp.  libstdc++ sifts the
// parents from (len - 2) / 2 down to 0; the parents of one depth have disjoint
// subtrees and all deeper parents come first, so each depth is sifted by the
// lanes at once.
template <class Cmp>
__device__ __forceinline__ void make_heap_warp(uint2* nd, int len, Cmp before) {
  const int lane = threadIdx.x & 31;
  if (len < 2) return;
  const int last_parent = (len - 2) / 2;
  for (int d = 31 - __clz(last_parent + 1); d >= 0; --d) {
    const int lo = (1 << d) - 1, hi = min(2 * lo, last_parent);  // parents of depth d
    for (int parent = hi - lane; parent >= lo; parent -= 32) sift_down(nd, parent, len, nd[parent + 1], before);
    __syncwarp();
  }
}

// Replacements of the heap select for the candidates list[0 .. m) (queue order),
// by one warp: candidate x replaces the top when it compares before it
// (__pop_heap + __adjust_heap).  The lanes test 32 candidates at a time against
// the top; lane 0 replays the replacements among them in order, re-testing each
// against its current top.  Returns the top.
template <class Cmp>
__device__ __forceinline__ uint32_t heap_replay(uint2* nd, int len, const uint2* list, int m, uint32_t top,
                                                Cmp before) {
  const int lane = threadIdx.x & 31;
  for (int base = 0; base < m; base += 32) {
    const int e = base + lane;
    const uint2 ce = e < m ? list[e] : make_uint2(0u, 0u);
    uint32_t hits = __ballot_sync(0xFFFFFFFFu, e < m && before(ce.x, top));
    if (hits) {
      if (lane == 0) {
        while (hits) {
          const int f = __ffs(hits) - 1;
          hits &= hits - 1;
          const uint2 x = list[base + f];
          if (before(x.x, top)) top = sift_down(nd, 0, len, x, before);
        }
      }
      top = __shfl_sync(0xFFFFFFFFu, top, 0);
    }
  }
  __syncwarp();
  return top;
}

// __heap_select(0, k, n) over the queue by the whole block.  The heap's nodes
// live in `nd` (at least k + 8 entries, 16-byte aligned); the queue after the
// first k entries is taken in windows of at most `lcap` (and kSelWindow) entries: the block
// copies the entries of a window that compare before the current top (the top
// only moves on, so no other entry of the window can replace it) into `list`,
// in queue order, and warp 0 replays them.  The first k queue entries receive
// the result; the evicted entries are not written back (nothing reads past the
// first k).
template <class Cmp>
__device__ __forceinline__ void heap_select_block(const Queue& Q, int k, int n, Cmp before, uint2* nd, uint2* list,
                                                  int lcap,
                                  SelShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) {
    for (int i = lane; i < k; i += 32) nd[i + 1] = make_uint2(Q.qk[i], (uint32_t)Q.q[i]);
    __syncwarp();
    make_heap_warp(nd, k, before);
    if (lane == 0) sh.pivot = nd[1].x;
  }
  __syncthreads();
  // Short windows keep the filter's top close to the replay's, so fewer entries
  // reach the list.
  lcap = min(lcap, kSelWindow);
  for (int lo = k; lo < n; lo += lcap) {
    const int hi = min(n, lo + lcap);
    const uint32_t top = sh.pivot;
    const Chunk rc = range_chunk(lo, hi, warp);
    uint32_t cnt = 0;
    for (int b = rc.begin; b < rc.end; b += 128) {
      uint32_t kk[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = b + 32 * j + lane;
        kk[j] = i < rc.end ? Q.qk[i] : 0u;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        cnt += __popc(__ballot_sync(0xFFFFFFFFu, b + 32 * j + lane < rc.end && before(kk[j], top)));
    }
    if (lane == 0) sh.warp_cnt[0][warp] = cnt;
    scan_warp_counts(sh, 1);
    uint32_t off = sh.warp_off[0][warp];
    const uint32_t below = (1u << lane) - 1u;
    for (int b = rc.begin; b < rc.end; b += 128) {
      uint32_t kk[4];
      int pp[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = b + 32 * j + lane;
        kk[j] = i < rc.end ? Q.qk[i] : 0u;
        pp[j] = i < rc.end ? Q.q[i] : 0;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool hit = b + 32 * j + lane < rc.end && before(kk[j], top);
        const uint32_t bal = __ballot_sync(0xFFFFFFFFu, hit);
        if (hit) list[off + __popc(bal & below)] = make_uint2(kk[j], (uint32_t)pp[j]);
        off += __popc(bal);
      }
    }
    const int m = (int)(sh.warp_off[0][kSelWarps - 1] + sh.warp_cnt[0][kSelWarps - 1]);
    __syncthreads();
    if (warp == 0) {
      const uint32_t t = heap_replay(nd, k, list, m, top, before);
      if (lane == 0) sh.pivot = t;
    }
    __syncthreads();
  }
  if (warp == 0) {
    for (int i = lane; i < k; i += 32) {
      const uint2 v = nd[i + 1];
      Q.qk[i] = v.x;
      Q.q[i] = (int)v.y;
    }
  }
  __syncthreads();
}

// __adjust_heap followed by __push_heap on the queue's heap [first, first + len),
// one thread (the introselect's depth-limit fallback).
__device__ void adjust_heap_queue(const Queue& Q, int first, int hole, int len, int item, uint32_t item_key,
                                  Before before) {
  int* q = Q.q + first;
  uint32_t* qk = Q.qk + first;
  const int top = hole;
  int child = hole;
  while (child < (len - 1) / 2) {
    child = 2 * (child + 1);
    if (before(qk[child], qk[child - 1])) --child;
    q[hole] = q[child];
    qk[hole] = qk[child];
    hole = child;
  }
  if ((len & 1) == 0 && child == (len - 2) / 2) {
    child = 2 * (child + 1);
    q[hole] = q[child - 1];
    qk[hole] = qk[child - 1];
    hole = child - 1;
  }
  int parent = (hole - 1) / 2;
  while (hole > top && before(qk[parent], item_key)) {
    q[hole] = q[parent];
    qk[hole] = qk[parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  q[hole] = item;
  qk[hole] = item_key;
}

// __heap_select(first, middle, last) in place, one thread.
__device__ void heap_select_serial(const Queue& Q, int first, int middle, int last, Before before) {
  const int len = middle - first;
  if (len >= 2)
    for (int parent = (len - 2) / 2;; --parent) {
      adjust_heap_queue(Q, first, parent, len, Q.q[first + parent], Q.qk[first + parent], before);
      if (parent == 0) break;
    }
  for (int i = middle; i < last; ++i) {
    const int item = Q.q[i];
    const uint32_t k = Q.qk[i];
    if (before(k, Q.qk[first])) {
      Q.q[i] = Q.q[first];
      Q.qk[i] = Q.qk[first];
      adjust_heap_queue(Q, first, 0, len, item, k, before);
    }
  }
}

// __insertion_sort(first, last), one thread.
__device__ void insertion_sort_serial(const Queue& Q, int first, int last, Before before) {
  for (int i = first + 1; i < last; ++i) {
    const int item = Q.q[i];
    const uint32_t k = Q.qk[i];
    int j = i;
    if (before(k, Q.qk[first])) {
      for (; j > first; --j) {
        Q.q[j] = Q.q[j - 1];
        Q.qk[j] = Q.qk[j - 1];
      }
    } else {
      while (before(k, Q.qk[j - 1])) {
        Q.q[j] = Q.q[j - 1];
        Q.qk[j] = Q.qk[j - 1];
        --j;
      }
    }
    Q.q[j] = item;
    Q.qk[j] = k;
  }
}


// Candidates (tier byte kCand) among tokens t0 .. t0 + 15 below `end`, as a bit
// mask (bit i: token t0 + i); t0 is a multiple of 16.
__device__ __forceinline__ uint32_t cand_mask16(const uint8_t* tier, int t0, int end) {
  uint32_t w[4] = {0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu};
  if (t0 + 16 <= end) {
    const uint4 v = *reinterpret_cast<const uint4*>(tier + t0);
    w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
  } else {
    for (int i = 0; i < 16 && t0 + i < end; ++i)
      w[i >> 2] = (w[i >> 2] & ~(0xFFu << (8 * (i & 3)))) | ((uint32_t)tier[t0 + i] << (8 * (i & 3)));
  }
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) m |= (((w[i >> 2] >> (8 * (i & 3))) & 0xFFu) == kCand ? 1u : 0u) << i;
  return m;
}

// Mark the k candidates torch.topk would choose, by one block over all T tokens
// (st: tier bytes of [0, T)).  The candidates are compacted into the queue in
// position order first, with their keys beside them.
template <bool SMEM>
__device__ void select_exact(const SelectParams& p, const SelState<SMEM>& st, const float* src, int k, bool largest,
                             uint8_t mark, SelShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const Queue Q{p.queue, p.qkey};
  const Before before{largest};
  // queue of candidates in position order: 16 tokens per lane per step (one
  // 16-byte load of tier bytes), the lanes' counts scanned across the warp
  const Chunk ch = warp_chunk(0, p.T, warp);  // starts at a multiple of 128
  uint32_t cnt = 0;
  for (int b = ch.begin; b < ch.end; b += 512) cnt += __popc(cand_mask16(st.tier, b + 16 * lane, ch.end));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, o);
  if (lane == 0) sh.warp_cnt[0][warp] = cnt;
  scan_warp_counts(sh, 1);
  uint32_t off = sh.warp_off[0][warp];
  const uint32_t below = (1u << lane) - 1u;
  for (int b = ch.begin; b < ch.end; b += 128) {  // coalesced stores: 32 tokens per ballot
    uint8_t tb[4];
    float sc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = b + 32 * j + lane;
      tb[j] = t < ch.end ? st.tier[t] : (uint8_t)0xFF;
      sc[j] = tb[j] == kCand ? src[t] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool c = tb[j] == kCand;
      const uint32_t bal = __ballot_sync(0xFFFFFFFFu, c);
      if (c) {
        const uint32_t pos = off + __popc(bal & below);
        Q.q[pos] = b + 32 * j + lane;
        Q.qk[pos] = order_key(sc[j]);
      }
      off += __popc(bal);
    }
  }
  const int n = (int)(sh.warp_off[0][kSelWarps - 1] + sh.warp_cnt[0][kSelWarps - 1]);
  __syncthreads();
  if (k > n) k = n;  // the count check reports the shortfall
  if (k <= 0) return;
  if ((int64_t)k * 64 <= n) {
    // Scratch: this block's dynamic shared memory (its own tokens' tier bytes
    // are in the workspace meanwhile; the caller restores its keys).  The heap
    // nodes go there when they leave room for a window of 4096 entries, else
    // into the stop table (k * 64 <= T: room for k + 8 nodes).
    extern __shared__ __align__(16) uint8_t sel_smem[];
    const size_t nb = heap_node_bytes(k);
    // (each call inlined with its nodes' memory space known to the compiler)
    if (nb + 8 * 4096 <= (size_t)p.smem_bytes) {
      uint2* const nd = reinterpret_cast<uint2*>(sel_smem);
      uint2* const list = reinterpret_cast<uint2*>(sel_smem + nb);
      const int lcap = (int)((p.smem_bytes - nb) / 8);
      if (largest) heap_select_block(Q, k, n, BeforeC<true>{}, nd, list, lcap, sh);
      else heap_select_block(Q, k, n, BeforeC<false>{}, nd, list, lcap, sh);
    } else {
      uint2* const nd = reinterpret_cast<uint2*>(p.stops);
      uint2* const list = reinterpret_cast<uint2*>(sel_smem);
      const int lcap = p.smem_bytes / 8;
      if (largest) heap_select_block(Q, k, n, BeforeC<true>{}, nd, list, lcap, sh);
      else heap_select_block(Q, k, n, BeforeC<false>{}, nd, list, lcap, sh);
    }
  } else {
    const int nth = k - 1;
    // Working copy: the queue in the workspace until the remaining range (with
    // its stop table, 12 bytes an entry) fits this block's shared memory, then
    // there (indices unchanged), copied back at the end.
    extern __shared__ __align__(16) uint8_t sel_smem[];
    Queue W = Q;
    int* stops = p.stops;
    int moved_first = 0, moved_last = 0;
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
      if (moved_last == 0 && (size_t)(last - first) * 12 + 16 <= (size_t)p.smem_bytes) {
        const int R = last - first;
        int* qs = reinterpret_cast<int*>(sel_smem);
        uint32_t* ks = reinterpret_cast<uint32_t*>(sel_smem + 4 * (size_t)R);
        for (int i = threadIdx.x; i < R; i += kSelThreads) {
          qs[i] = Q.q[first + i];
          ks[i] = Q.qk[first + i];
        }
        W = Queue{qs - first, ks - first};
        stops = reinterpret_cast<int*>(sel_smem + 8 * (size_t)R);
        moved_first = first;
        moved_last = last;
        __syncthreads();
      }
      if (depth == 0) {
        if (threadIdx.x == 0) {
          heap_select_serial(W, first, nth + 1, last, before);
          W.swap(first, nth);
          sh.done = 2;
        }
        break;
      }
      if (threadIdx.x == 0) {
        sh.depth = depth - 1;
        const int a = first + 1, b = first + (last - first) / 2, c = last - 1;
        const uint32_t ka = W.qk[a], kb = W.qk[b], kc = W.qk[c];
        int m;
        uint32_t km;
        if (before(ka, kb)) {
          if (before(kb, kc)) m = b, km = kb;
          else if (before(ka, kc)) m = c, km = kc;
          else m = a, km = ka;
        } else if (before(ka, kc)) {
          m = a, km = ka;
        } else if (before(kb, kc)) {
          m = c, km = kc;
        } else {
          m = b, km = kb;
        }
        W.swap(first, m);
        sh.pivot = km;
        sh.pairs = 0;
      }
      __syncthreads();
      const uint32_t piv = sh.pivot;
      const int lo = first + 1, hi = last;
      // Stop tables: at most (hi - lo) / 2 swaps, so left stops of rank <= H and
      // right stops of rank < H are all that is read; they share one region.
      const int H = (hi - lo) / 2;
      int* const stop_l = stops;
      int* const stop_r = stops + H + 1;
      const Chunk rc = range_chunk(lo, hi, warp);
      // pass 1: left / right stops per warp piece
      uint32_t nl = 0, nr = 0;
      for (int b = rc.begin; b < rc.end; b += 128) {
        uint32_t kk[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = b + 32 * j + lane;
          kk[j] = i < rc.end ? W.qk[i] : 0u;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool valid = b + 32 * j + lane < rc.end;
          nl += __popc(__ballot_sync(0xFFFFFFFFu, valid && !before(kk[j], piv)));
          nr += __popc(__ballot_sync(0xFFFFFFFFu, valid && !before(piv, kk[j])));
        }
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
      const uint32_t below = (1u << lane) - 1u;
      for (int b = rc.begin; b < rc.end; b += 128) {
        uint32_t kk[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = b + 32 * j + lane;
          kk[j] = i < rc.end ? W.qk[i] : 0u;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = b + 32 * j + lane;
          const bool valid = i < rc.end;
          const bool ls = valid && !before(kk[j], piv), rs = valid && !before(piv, kk[j]);
          const uint32_t bl = __ballot_sync(0xFFFFFFFFu, ls), br = __ballot_sync(0xFFFFFFFFu, rs);
          const int lrank = (int)(left_before + __popc(bl & below));     // left stops in [lo, i)
          const int rbefore = (int)(right_before + __popc(br & below));  // right stops in [lo, i)
          const int ri = total_r - 1 - rbefore;
          if (ls && lrank <= H) stop_l[lrank] = i;
          if (rs && ri < H) stop_r[ri] = i;
          if (valid) best = max(best, min(lrank, total_r - rbefore));  // cut just before slot i
          left_before += __popc(bl);
          right_before += __popc(br);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
      if (lane == 0 && best > 0) atomicMax(&sh.pairs, best);
      __syncthreads();
      const int pairs = sh.pairs;
      // pass 3: the swaps (disjoint slot pairs)
      for (int m0 = threadIdx.x; m0 < pairs; m0 += 4 * kSelThreads) {  // four swaps in flight
        int li[4], ri[4], a[4], b[4];
        uint32_t ka[4], kb[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int m = m0 + u * kSelThreads;
          li[u] = m < pairs ? stop_l[m] : -1;
          ri[u] = m < pairs ? stop_r[m] : -1;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (li[u] >= 0) {
            a[u] = W.q[li[u]], b[u] = W.q[ri[u]];
            ka[u] = W.qk[li[u]], kb[u] = W.qk[ri[u]];
          }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (li[u] >= 0) {
            W.q[li[u]] = b[u], W.q[ri[u]] = a[u];
            W.qk[li[u]] = kb[u], W.qk[ri[u]] = ka[u];
          }
      }
      if (threadIdx.x == 0) {
        int cut = -1;
        if (pairs >= 1 && !(pairs < total_l && stop_l[pairs] < stop_r[pairs - 1])) cut = stop_r[pairs - 1];
        else if (pairs < total_l) cut = stop_l[pairs];
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
    if (threadIdx.x == 0 && sh.done == 0) insertion_sort_serial(W, sh.first, sh.last, before);
    __syncthreads();
    for (int i = moved_first + (int)threadIdx.x; i < moved_last; i += kSelThreads) {
      Q.q[i] = W.q[i];
      Q.qk[i] = W.qk[i];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < k; i += kSelThreads) st.tier[Q.q[i]] = mark;
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Radix selection.  The k-th key is found one digit at a time from the top
// (bits [21,32), [10,21), [0,10)): each block counts the digit over its own
// candidates that match the digits found so far, and after a cluster barrier
// every block sums the eight histograms and scans them in rank order for the bin
// holding the k-th candidate.  The count in the last bin is the number of
// candidates equal to the k-th key, so the tie test needs no pass of its own.
// Without a tie the selection is "every candidate at or beyond the k-th key";
// that mark is not written at once but applied by the next sweep (the first
// digit of the next selection, or the count of the final compaction).
// ---------------------------------------------------------------------------

// A finished selection whose marks the next sweep applies.
struct MarkOp {
  const float* src;  // keys: nullptr = importance scores (cached in SMEM mode)
  uint32_t tau;      // k-th key
  uint8_t mark;
  bool largest;
  bool on;
};
__device__ __forceinline__ MarkOp no_mark() { return MarkOp{nullptr, 0u, 0, false, false}; }
__device__ __forceinline__ bool takes(const MarkOp& m, uint32_t key) {
  return m.largest ? key >= m.tau : key <= m.tau;
}

__device__ __forceinline__ int digit_shift(int d) { return d == 0 ? 21 : (d == 1 ? 10 : 0); }
__device__ __forceinline__ int digit_bins(int d) { return d == 2 ? 1024 : 2048; }
// bits above digit d
__device__ __forceinline__ uint32_t high_mask(int d) { return d == 0 ? 0u : (d == 1 ? 0xFFE00000u : 0xFFFFFC00u); }

// Warp-aggregated histogram increment: one shared atomic per distinct digit.
__device__ __forceinline__ void hist_add(uint32_t* hist, bool act, uint32_t digit) {
  const uint32_t am = __ballot_sync(0xFFFFFFFFu, act);
  if (act) {
    const uint32_t peers = __match_any_sync(am, digit);
    if ((threadIdx.x & 31) == (unsigned)(__ffs(peers) - 1)) atomicAdd(&hist[digit], __popc(peers));
  }
}

struct BinPick {
  uint32_t bin, remaining, count;
  bool found;
};

// Bin of the rem-th candidate in rank order (descending digits for `largest`)
// over the cluster's histograms hist[buf], the rank left inside it and its count.
// Call after the cluster barrier that follows the counting; every block computes
// the same pick, which returns to every thread.
__device__ BinPick find_bin(SelShared& sh, int buf, int nbins, uint32_t rem, bool largest) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per = nbins / kSelThreads;  // 1 or 2 scan positions per thread
  uint32_t c[2] = {0u, 0u}, sum = 0;
#pragma unroll
  for (int j = 0; j < 2; ++j)
    if (j < per) {
      const int pos = threadIdx.x * per + j;
      uint32_t* const h = &sh.hist[buf][largest ? nbins - 1 - pos : pos];
      uint32_t v[kSelCluster];
#pragma unroll
      for (int r = 0; r < kSelCluster; ++r) v[r] = ld_peer(h, r);
#pragma unroll
      for (int r = 0; r < kSelCluster; ++r) c[j] += v[r];
      sum += c[j];
    }
  uint32_t inc = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) sh.wsum[warp] = inc;
  if (threadIdx.x == 0) sh.found = 0;
  __syncthreads();
  uint32_t winc = sh.wsum[lane];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, winc, o);
    if (lane >= o) winc += t;
  }
  const uint32_t wpre = __shfl_sync(0xFFFFFFFFu, winc, (warp + 31) & 31);
  const uint32_t before = (warp ? wpre : 0u) + inc - sum;
  if (before < rem && before + sum >= rem) {  // exactly one thread when rem <= total
    uint32_t cum = before;
    int j = 0;
    if (per == 2 && cum + c[0] < rem) {
      cum += c[0];
      j = 1;
    }
    const int pos = threadIdx.x * per + j;
    sh.pick_bin = (uint32_t)(largest ? nbins - 1 - pos : pos);
    sh.pick_rem = rem - cum;
    sh.pick_cnt = j ? c[1] : c[0];
    sh.found = 1;
  }
  __syncthreads();
  return BinPick{sh.pick_bin, sh.pick_rem, sh.pick_cnt, sh.found != 0};
}

// Sweep of this block's tokens: apply the pending marks `pm`, then count digit d
// of the candidates' keys (src) that match `prefix` above it into `hist`.  INIT:
// the sweep also writes the initial tiers (sink and tail retained) and, in SMEM
// mode, the cached keys of the importance scores.
template <bool SMEM, bool INIT>
__device__ void hist_sweep(const SelectParams& p, const SelState<SMEM>& st, uint32_t* hist, const MarkOp& pm,
                           const float* src, int d, uint32_t prefix) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int shift = digit_shift(d);
  const uint32_t dmask = (uint32_t)digit_bins(d) - 1u, hmask = high_mask(d);
  const Chunk ch = warp_chunk(st.base, st.end, warp);
  for (int b = ch.begin; b < ch.end; b += 4 * 32) {
    uint8_t tr[4];
    uint32_t own[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = b + 32 * j + lane;
      tr[j] = 0xFF;
      own[j] = 0u;
      if (t < ch.end) {
        if (INIT) {
          tr[j] = (t < p.sink || t >= p.T - p.tail) ? kRet : kCand;
          if (SMEM && p.scores) own[j] = order_key(p.scores[t]);
        } else {
          tr[j] = st.tier[t - st.base];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = b + 32 * j + lane;
      if (t < ch.end) {
        if (INIT && SMEM && p.scores) st.keys[t - st.base] = own[j];
        bool store = INIT;
        if (pm.on && tr[j] == kCand && takes(pm, key_at<SMEM>(st, pm.src, t))) {
          tr[j] = pm.mark;
          store = true;
        }
        if (store) st.tier[t - st.base] = tr[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = b + 32 * j + lane;
      bool act = false;
      uint32_t digit = 0;
      if (tr[j] == kCand) {
        const uint32_t key = (INIT && SMEM && src == nullptr && p.scores) ? own[j] : key_at<SMEM>(st, src, t);
        if ((key & hmask) == prefix) {
          act = true;
          digit = (key >> shift) & dmask;
        }
      }
      hist_add(hist, act, digit);
    }
  }
}

// A tie across the boundary: block 0 runs select_exact over the tier bytes of
// all T tokens in global memory (SMEM mode: every block copies its own out and
// back around it).
template <bool SMEM>
__device__ void exact_on_block0(const SelectParams& p, const SelState<SMEM>& st, SelShared& sh, const float* src,
                                int k, bool largest, uint8_t mark) {
  if (SMEM)
    for (int t = st.base + (int)threadIdx.x; t < st.end; t += kSelThreads) p.tier[t] = st.tier[t - st.base];
  cluster_sync();
  if (cg::this_cluster().block_rank() == 0) {
    const SelState<false> all{nullptr, p.tier, 0, p.T};
    select_exact<false>(p, all, src ? src : p.scores, k, largest, mark, sh);
    if (SMEM && p.scores)  // the exact path used the cached keys' shared memory as scratch
      for (int t = st.base + (int)threadIdx.x; t < st.end; t += kSelThreads)
        st.keys[t - st.base] = order_key(p.scores[t]);
  }
  cluster_sync();
  if (SMEM) {
    for (int t = st.base + (int)threadIdx.x; t < st.end; t += kSelThreads) st.tier[t - st.base] = p.tier[t];
    __syncthreads();
  }
}

// Select the k candidates (tier == kCand) with the largest (smallest) keys of
// `src` and return their mark for the next sweep; a tie across the boundary is
// resolved and marked here.  `pm`: the previous selection's pending marks,
// applied by the first-digit sweep.  `buf`: histogram buffer of the next pass.
// save: keep this selection's first-digit counts (hist[2]) and bin for a later
// selection over the same keys.  from_saved: a smallest-k selection that may take
// its first digit from those counts: the earlier (largest-k) selection marks only
// candidates in its bin or above, so the counts below that bin are this
// selection's too; when the k-th smallest lies below it, the first sweep is
// skipped and the pending marks ride with the second.
template <bool SMEM>
__device__ MarkOp select_radix(const SelectParams& p, const SelState<SMEM>& st, SelShared& sh, const MarkOp& pm,
                               bool init, const float* src, int k, bool largest, uint8_t mark, int& buf,
                               bool save = false, bool from_saved = false) {
  BinPick bp{0u, (uint32_t)k, 0u, true};
  uint32_t prefix = 0u;
  int d0 = 0;
  MarkOp first_pm = pm;
  if (save && threadIdx.x == 0) sh.saved_bin = 0;  // no reuse unless the first digit is found
  if (from_saved && !largest) {
    const BinPick sb = find_bin(sh, 2, digit_bins(0), (uint32_t)k, false);
    if (sb.found && sb.bin < sh.saved_bin) {
      bp = sb;
      prefix = sb.bin << digit_shift(0);
      d0 = 1;
    }
  }
  for (int d = d0; d < 3; ++d) {
    for (int i = threadIdx.x; i < kBins; i += kSelThreads) sh.hist[buf][i] = 0;
    __syncthreads();
    if (d == 0 && init) hist_sweep<SMEM, true>(p, st, sh.hist[buf], pm, src, 0, 0u);
    else hist_sweep<SMEM, false>(p, st, sh.hist[buf], d == d0 ? first_pm : no_mark(), src, d, prefix);
    if (save && d == 0) {
      __syncthreads();
      for (int i = threadIdx.x; i < kBins; i += kSelThreads) sh.hist[2][i] = sh.hist[buf][i];
    }
    cluster_sync();
    bp = find_bin(sh, buf, digit_bins(d), bp.remaining, largest);
    buf ^= 1;
    // fewer candidates than k: mark all of them; the final count check reports it
    if (!bp.found) return MarkOp{src, largest ? 0u : 0xFFFFFFFFu, mark, largest, true};
    if (save && d == 0 && threadIdx.x == 0) sh.saved_bin = bp.bin;
    prefix |= bp.bin << digit_shift(d);
  }
  if (bp.remaining < bp.count) {  // candidates equal to the k-th key straddle the boundary
    exact_on_block0<SMEM>(p, st, sh, src, k, largest, mark);
    return no_mark();
  }
  return MarkOp{src, prefix, mark, largest, true};
}

// Apply the last pending marks and write the three ascending index lists.
template <bool SMEM>
__device__ void compact_lists(const SelectParams& p, const SelState<SMEM>& st, SelShared& sh, const MarkOp& pm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const Chunk ch = warp_chunk(st.base, st.end, warp);
  uint32_t n_ret = 0, n_cold = 0, n_all = 0;
  for (int b = ch.begin; b < ch.end; b += 4 * 32) {
    uint8_t tr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = b + 32 * j + lane;
      tr[j] = t < ch.end ? st.tier[t - st.base] : 0xFF;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = b + 32 * j + lane;
      if (pm.on && tr[j] == kCand && takes(pm, key_at<SMEM>(st, pm.src, t))) {
        tr[j] = pm.mark;
        st.tier[t - st.base] = tr[j];
      }
      n_ret += tr[j] == kRet;
      n_cold += tr[j] == kCold;
      n_all += tr[j] != 0xFF;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    n_ret += __shfl_xor_sync(0xFFFFFFFFu, n_ret, o);
    n_cold += __shfl_xor_sync(0xFFFFFFFFu, n_cold, o);
    n_all += __shfl_xor_sync(0xFFFFFFFFu, n_all, o);
  }
  if (lane == 0) {
    sh.warp_cnt[0][warp] = n_ret;
    sh.warp_cnt[1][warp] = n_all - n_ret - n_cold;
    sh.warp_cnt[2][warp] = n_cold;
  }
  scan_warp_counts(sh, 3);
  if (threadIdx.x < 3) sh.list_tot[threadIdx.x] = sh.warp_off[threadIdx.x][kSelWarps - 1] +
                                                  sh.warp_cnt[threadIdx.x][kSelWarps - 1];
  cluster_sync();
  if (threadIdx.x < 3) {
    const int rank = (int)cg::this_cluster().block_rank();
    uint32_t below = 0, all = 0;
    for (int r = 0; r < kSelCluster; ++r) {
      const uint32_t v = ld_peer(&sh.list_tot[threadIdx.x], r);
      below += r < rank ? v : 0u;
      all += v;
    }
    sh.list_off[threadIdx.x] = below;
    sh.list_all[threadIdx.x] = all;
  }
  cluster_sync();  // peers' counts read before any block moves on (and exits)
  uint32_t off_r = sh.list_off[0] + sh.warp_off[0][warp], off_s = sh.list_off[1] + sh.warp_off[1][warp],
           off_c = sh.list_off[2] + sh.warp_off[2][warp];
  const uint32_t below = (1u << lane) - 1u;
  for (int b = ch.begin; b < ch.end; b += 4 * 32) {
    uint8_t tr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = b + 32 * j + lane;
      tr[j] = t < ch.end ? st.tier[t - st.base] : 0xFF;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = b + 32 * j + lane;
      const uint32_t br = __ballot_sync(0xFFFFFFFFu, tr[j] == kRet);
      const uint32_t bs = __ballot_sync(0xFFFFFFFFu, tr[j] == kCand);
      const uint32_t bc = __ballot_sync(0xFFFFFFFFu, tr[j] == kCold);
      if (tr[j] == kRet) {
        const uint32_t pos = off_r + __popc(br & below);
        if (pos < (uint32_t)p.n_ret) p.idx_ret[pos] = t;
      } else if (tr[j] == kCand) {
        const uint32_t pos = off_s + __popc(bs & below);
        if (pos < (uint32_t)p.n_std) p.idx_std[pos] = t;
      } else if (tr[j] == kCold) {
        const uint32_t pos = off_c + __popc(bc & below);
        if (pos < (uint32_t)p.n_cold) p.idx_cold[pos] = t;
      }
      off_r += __popc(br);
      off_s += __popc(bs);
      off_c += __popc(bc);
    }
  }
  if (threadIdx.x == 0 && cg::this_cluster().block_rank() == 0) {
    if (sh.list_all[0] != (uint32_t)p.n_ret || sh.list_all[1] != (uint32_t)p.n_std ||
        sh.list_all[2] != (uint32_t)p.n_cold)
      raise_error(kErrSelectCount);
  }
}

template <bool SMEM>
__device__ void select_body(const SelectParams& p, SelState<SMEM> st, SelShared& sh) {
  const float* const scores_src = SMEM ? nullptr : p.scores;
  MarkOp pm = no_mark();
  bool init = true;
  int buf = 0;
  // the cold tier may reuse the protection's first digit (same keys, no outlier
  // selection in between)
  const bool reuse = p.keep_protect > 0 && p.keep_outlier == 0 && p.keep_cold > 0;
  if (p.keep_protect > 0) {
    pm = select_radix<SMEM>(p, st, sh, pm, init, scores_src, p.keep_protect, true, kRet, buf, reuse);
    init = false;
  }
  if (p.keep_outlier > 0) {
    pm = select_radix<SMEM>(p, st, sh, pm, init, p.outlier, p.keep_outlier, true, kRet, buf);
    init = false;
  }
  if (p.keep_cold > 0) {
    pm = select_radix<SMEM>(p, st, sh, pm, init, scores_src, p.keep_cold, false, kCold, buf, false, reuse);
    init = false;
  }
  if (init) {  // no score selection: sink and tail only
    for (int t = st.base + (int)threadIdx.x; t < st.end; t += kSelThreads)
      st.tier[t - st.base] = (t < p.sink || t >= p.T - p.tail) ? kRet : kCand;
  }
  __syncthreads();
  compact_lists<SMEM>(p, st, sh, pm);
}

// Tokens per block of the selection cluster (a multiple of 128).
__host__ __device__ __forceinline__ int select_block_tokens(int T) {
  return ((T + kSelCluster - 1) / kSelCluster + 127) & ~127;
}

__global__ void __cluster_dims__(kSelCluster, 1, 1) __launch_bounds__(kSelThreads, 1)
    select_kernel(const SelectParams p) {
  __shared__ SelShared sh;
  extern __shared__ __align__(16) uint8_t sel_smem[];
  const int per = select_block_tokens(p.T);
  const int base = min(p.T, (int)cg::this_cluster().block_rank() * per), end = min(p.T, base + per);
  if (per <= kSelSmemTokens) {
    SelState<true> st{reinterpret_cast<uint32_t*>(sel_smem), sel_smem + 4 * (size_t)per, base, end};
    select_body<true>(p, st, sh);
  } else {
    SelState<false> st{nullptr, p.tier + base, base, end};
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

// Workspace of the select kernel: tier bytes [T], then the queue's positions and
// keys (4 bytes [T] each) and the stop tables (int32 [T + 1]), every region
// 256-byte aligned.
constexpr size_t select_region(int T) { return ((size_t)T * 4 + 255) & ~(size_t)255; }
constexpr size_t select_workspace(int T) {
  return (((size_t)T + 255) & ~(size_t)255) + 2 * select_region(T) + select_region(T + 1);
}

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
  p.qkey = reinterpret_cast<uint32_t*>(w + select_region(T));
  p.stops = reinterpret_cast<int*>(w + 2 * select_region(T));
  p.idx_ret = idx_ret;
  p.idx_std = idx_std;
  p.idx_cold = idx_cold;
  // The blocks' own tokens (kSelSmemTokens * 5 bytes at most, below the limit
  // with the static part rounded up to 1 KB), and at least kSelExactSmem for the
  // exact path's scratch in block 0 (its tokens' space included).
  constexpr size_t kStatic = (sizeof(SelShared) + 1023) & ~(size_t)1023;
  static_assert(kSelSmemLimit - kStatic >= (size_t)kSelSmemTokens * 5, "select smem");
  const int per = select_block_tokens(T);
  const size_t sm = std::max(per <= kSelSmemTokens ? (size_t)per * 5 : (size_t)0, kSelExactSmem);
  p.smem_bytes = (int)sm;
  cudaError_t e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  select_kernel<<<kSelCluster, kSelThreads, sm, st>>>(p);
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
