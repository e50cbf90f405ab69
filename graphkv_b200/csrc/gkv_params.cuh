// Launch parameters resolved on the host from a gkv_plan (passed by value as
// __grid_constant__ kernel arguments, kept under the classic 4 KiB limit).
#pragma once

#include "gkv_common.cuh"

namespace gkv {

constexpr int kThreads = 256;    // threads per block of the tile kernels
constexpr int kMaxLayers = 40;   // layers per launch (larger calls are split)
constexpr int kRetTile = 64;     // retained rows per tile
constexpr int kRun = 32;         // elements of one thread's run along the grouped axis (tile kernels)
constexpr int kTokRun = 16;      // rows of one thread's run of a token-axis quantizer

// Tier numbering inside the kernels: 0 retained, 1 standard, 2 cold.
// Tensor numbering follows gkv_tensor_slot: 0 std K, 1 std V, 2 cold K, 3 cold V.

// Division of 32-bit unsigned integers by a divisor fixed per launch: the
// round-up multiply-high method of T. Granlund and P. Montgomery ("Division by
// invariant integers using multiplication", PLDI 1994, figure 4.1), exact for
// every n < 2^32 and 1 <= d <= 2^31.
struct FastDiv {
  uint32_t d, m;
  int s1, s2;
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    const uint32_t t = __umulhi(m, n);
    return (t + ((n - t) >> s1)) >> s2;
  }
};
inline FastDiv make_fastdiv(uint32_t d) {
  int l = 0;
  while ((1ull << l) < d) ++l;
  FastDiv f;
  f.d = d;
  f.m = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
  f.s1 = l > 0 ? 1 : 0;
  f.s2 = l > 0 ? l - 1 : 0;
  return f;
}

struct TensorDesc {
  int bits;         // 2, 4, 8
  int quantizer;    // GKV_SYMMETRIC / GKV_AFFINE
  int axis;         // GKV_AXIS_TOKEN / GKV_AXIS_CHANNEL
  int gs;           // effective group size
  int log2gs;       // log2(gs) when gs is a power of two, else -1
  int rotation;     // GKV_ROT_*
  int packed;       // 1: sub-byte packing
  int sbits;        // stored bits per code (bits when packed, else 8)
  int scale_dtype;  // GKV_F16 / GKV_BF16 / GKV_F32
  float qmax;       // largest code: 2^(bits-1) - 1 (symmetric) or 2^bits - 1 (affine)
  float rqmax;      // 1 / qmax rounded to nearest
  int n;            // tier length
  int n_pad;        // token axis: padded tier length; channel axis: padded head_dim
  int groups_row;   // token axis: groups per channel (n_pad / gs); channel: groups per token
  int64_t elems_slice;   // codes per slice
  int64_t groups_slice;  // groups per slice
  uint8_t* codes;
  void* scales;
  uint8_t* zps;     // affine only
  float* scale32;   // general path workspace: fp32 coding scales per group
  void* rot;        // general path workspace: rotated tier rows [S, n, D]
};

struct LayerDesc {
  const void* k;
  const void* v;
  int64_t ks[3];    // batch, head, token strides (elements)
  int64_t vs[3];
  int heads;
  int slice_begin;  // first slice of this layer within the launch
};

struct QuantParams {
  int B, T, D, S, n_layers;
  const int* idx[3];
  int n_tier[3];
  TensorDesc t[4];
  void* ret_k;
  void* ret_v;
  float had_div, had_inv;
  int had_fused;     // 1: had_div is fp32(sqrt(D)) with the fused quotient proven exact for it
  int tt;            // tile rows of the fast path (64 or 128)
  int tiles[3];      // fast-path tiles per slice per tier (0 when the tier is not in this launch)
  int tiles_slice;
  int slice_offset;  // global index of slice 0 of this launch (retained / codes addressing)
  FastDiv tile_div;  // by tiles_slice
  FastDiv layer_div; // by the slices of one layer when every layer has as many (d == 0: they differ)
  FastDiv head_div;  // by the heads of a layer (valid when layer_div is)
  LayerDesc layers[kMaxLayers];
};

int device_sm_count();  // host: SMs of the current device

struct DequantParams {
  int T, D, S;
  int out_T;         // tokens between two output slices (>= T)
  const int* idx[3];
  int n_tier[3];
  TensorDesc t[4];
  const void* ret_k;
  const void* ret_v;
  void* out_k;       // [S, out_T, D]
  void* out_v;
  float had_div, had_inv;
  int had_fused;     // as in QuantParams
  int tt;
  int tiles[3];
  int tiles_slice;
  FastDiv tile_div;  // by tiles_slice
};

// Params restricted to some tiers: the tile counts of the others are zeroed, so
// a launch's blocks map onto exactly the included tiers' tiles.
template <typename P>
P tiers_only(const P& p, bool retained, bool standard, bool cold) {
  P q = p;
  q.tiles[0] = retained ? p.tiles[0] : 0;
  q.tiles[1] = standard ? p.tiles[1] : 0;
  q.tiles[2] = cold ? p.tiles[2] : 0;
  q.tiles_slice = q.tiles[0] + q.tiles[1] + q.tiles[2];
  q.tile_div = make_fastdiv((uint32_t)(q.tiles_slice > 0 ? q.tiles_slice : 1));
  return q;
}

// Variant of a tier's tensor: 2 * axis + rotation (0..3).
inline int tier_variant(const TensorDesc& d) { return 2 * d.axis + (d.rotation ? 1 : 0); }

// Slice -> layer lookup (layers sorted by slice_begin).
__device__ __forceinline__ int find_layer(const QuantParams& p, int s) {
  if (p.layer_div.d) return (int)p.layer_div.div((uint32_t)s);
  int l = 0;
  while (l + 1 < p.n_layers && s >= p.layers[l + 1].slice_begin) ++l;
  return l;
}

}  // namespace gkv
