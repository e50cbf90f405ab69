// extern "C" entry points of libgraphkv_b200.so (declared in include/graphkv_b200.h):
// argument validation, routing of each tier to the tile kernels or the general
// kernels, workspace layout, and launches.  Nothing here allocates device memory.
// The library is one translation unit: the kernel sources are included below.
#include <atomic>
#include <mutex>
#include <cmath>
#include <cstdio>
#include <string>

#include "attention.cuh"
#include "dequantize.cuh"
#include "gkv_params.cuh"
#include "quantize.cuh"
#include "scores.cuh"
#include "select.cuh"

namespace gkv {

// Multiprocessor count of the current device (cached per device; host threads
// may race to fill an entry, and they all store the same value).
int device_sm_count() {
  static std::atomic<int> counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = counts[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

namespace {

thread_local std::string g_last_error;

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(GKV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool is_pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }
int ilog2(int x) { int l = 0; while ((1 << l) < x) ++l; return l; }
int elem_size(int dtype) { return dtype == GKV_F32 ? 4 : 2; }

// tile-kernel instantiations: (D, TT) per element size
bool tile_instantiated(int esize, int D, int TT) {
  (void)esize;
  return (D == 64 || D == 128) && (TT == 64 || TT == 128);
}

const int kTierOf[4] = {1, 1, 2, 2};

// A second stream per device on which the rotated value tiles are quantized and
// dequantized beside the key and plain value tiles of the caller's stream: the
// rotated kernels are bound by instruction issue and the others by memory, so
// they share the SMs well (measured on the 32k cache: quantize 0.539 -> 0.522 ms,
// dequant 0.518 -> 0.509 ms).  The helper stream starts after the caller's
// earlier work (fork event) and the caller's stream continues after the
// helper's kernels (join event).  The lock keeps one call's fork ... join
// sequence together when host threads overlap, so the helper holds only that
// call's kernels between its two events.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_side_mutex;
SideStream g_side[64];
constexpr int64_t kSideMinTiles = 8192;  // calls with fewer tiles stay on one stream

class SideStreamCall {
 public:
  // use: false runs everything on `st` (small calls, where the two event waits
  // cost more than the overlap gains).
  SideStreamCall(cudaStream_t st, bool use) : st_(st), lock_(g_side_mutex, std::defer_lock) {
    if (!use) return;
    lock_.lock();
    int dev = 0;
    if ((err_ = cudaGetDevice(&dev)) != cudaSuccess) return;
    if (dev < 0 || dev >= 64) {
      err_ = cudaErrorInvalidDevice;
      return;
    }
    SideStream& ss = g_side[dev];
    if (!ss.s) {
      if ((err_ = cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking)) != cudaSuccess) return;
      if ((err_ = cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming)) != cudaSuccess) return;
      if ((err_ = cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming)) != cudaSuccess) return;
    }
    if ((err_ = cudaEventRecord(ss.fork, st)) != cudaSuccess) return;
    if ((err_ = cudaStreamWaitEvent(ss.s, ss.fork, 0)) != cudaSuccess) return;
    side_ = &ss;
  }
  cudaStream_t side() const { return side_ ? side_->s : st_; }
  cudaError_t error() const { return err_; }
  // The caller's stream waits for the helper's kernels (also after a failed launch).
  cudaError_t join() {
    if (!side_ || joined_) return cudaSuccess;
    joined_ = true;
    cudaError_t e = cudaEventRecord(side_->join, side_->s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st_, side_->join, 0);
    return e;
  }
  ~SideStreamCall() { join(); }

 private:
  cudaStream_t st_;
  std::unique_lock<std::mutex> lock_;
  SideStream* side_ = nullptr;
  cudaError_t err_ = cudaSuccess;
  bool joined_ = false;
};

struct Resolved {
  TensorDesc t[4];
  int n[3];
  bool fast[3];   // [0]: retained copy inside the tile kernel; [1], [2]: tiers
  int tt;
  size_t ws_scale[4], ws_rot[4], ws_bytes;
};

int resolve_tensor(const gkv_plan& p, int i, int n, TensorDesc& d) {
  const gkv_tensor_spec& sp = p.spec[i];
  char buf[160];
  if (sp.bits != 2 && sp.bits != 4 && sp.bits != 8) {
    std::snprintf(buf, sizeof buf, "tensor %d: bits must be 2, 4 or 8 (got %d)", i, sp.bits);
    return fail(GKV_ERR_INVALID, buf);
  }
  if (sp.quantizer != GKV_SYMMETRIC && sp.quantizer != GKV_AFFINE) return fail(GKV_ERR_INVALID, "bad quantizer");
  if (sp.axis != GKV_AXIS_TOKEN && sp.axis != GKV_AXIS_CHANNEL) return fail(GKV_ERR_INVALID, "bad axis");
  if (sp.rotation != GKV_ROT_NONE && sp.rotation != GKV_ROT_HADAMARD) return fail(GKV_ERR_INVALID, "bad rotation");
  if (sp.scale_dtype < GKV_F32 || sp.scale_dtype > GKV_BF16) return fail(GKV_ERR_INVALID, "bad scale dtype");
  if (sp.packed && sp.bits == 8) return fail(GKV_ERR_INVALID, "8-bit codes are never packed");
  const int D = p.head_dim;
  const int axis_len = sp.axis == GKV_AXIS_TOKEN ? n : D;
  if (sp.group_size < 1 || sp.group_size > axis_len) {
    std::snprintf(buf, sizeof buf, "tensor %d: group_size %d outside [1, %d]", i, sp.group_size, axis_len);
    return fail(GKV_ERR_INVALID, buf);
  }
  if (sp.rotation && (!is_pow2(D) || D > 1024))
    return fail(GKV_ERR_INVALID, "hadamard rotation requires a power-of-two head dimension (<= 1024).");
  if (!p.codes[i] || !p.scales[i]) return fail(GKV_ERR_INVALID, "missing codes/scales storage");
  if (sp.quantizer == GKV_AFFINE && !p.zero_points[i]) return fail(GKV_ERR_INVALID, "affine tensor needs zero points");
  d.bits = sp.bits;
  d.quantizer = sp.quantizer;
  d.axis = sp.axis;
  d.gs = sp.group_size;
  d.log2gs = is_pow2(d.gs) ? ilog2(d.gs) : -1;
  d.rotation = sp.rotation;
  d.packed = sp.packed ? 1 : 0;
  d.sbits = d.packed ? d.bits : 8;
  d.scale_dtype = sp.scale_dtype;
  {
    const int qmax = sp.quantizer == GKV_AFFINE ? (1 << sp.bits) - 1 : (1 << (sp.bits - 1)) - 1;
    d.qmax = (float)qmax;
    d.rqmax = 1.0f / (float)qmax;  // IEEE single division: the correctly rounded reciprocal
  }
  d.n = n;
  const int len = axis_len;
  d.n_pad = (int)(ceil_div(len, d.gs) * d.gs);
  d.groups_row = d.n_pad / d.gs;
  if (sp.axis == GKV_AXIS_TOKEN) {
    d.elems_slice = (int64_t)D * d.n_pad;
    d.groups_slice = (int64_t)D * d.groups_row;
  } else {
    d.elems_slice = (int64_t)n * d.n_pad;
    d.groups_slice = (int64_t)n * d.groups_row;
  }
  d.codes = p.codes[i];
  d.scales = p.scales[i];
  d.zps = sp.quantizer == GKV_AFFINE ? p.zero_points[i] : nullptr;
  d.scale32 = nullptr;
  d.rot = nullptr;
  return GKV_OK;
}

// Can tensor d run in the tile kernels (tiles of 64 tier rows)?  Token-axis
// groups of 32 or 64 rows (a thread holds a column over a whole group);
// channel-axis groups are powers of two >= 32 dividing head_dim.  Rotated
// token-axis tensors dequantize on the general path.
bool tensor_fast(const TensorDesc& d, int esize, int D, int TT, bool quantize) {
  (void)esize;
  (void)TT;
  if (d.log2gs < 0 || d.gs < 32 || !aligned16(d.codes)) return false;
  if (d.axis == GKV_AXIS_TOKEN) return (d.gs == 32 || d.gs == 64) && (quantize || !d.rotation);
  return D % d.gs == 0;
}

bool layers_aligned(const gkv_layer_in* layers, int n_layers, int esize) {
  for (int l = 0; l < n_layers; ++l) {
    const gkv_layer_in& L = layers[l];
    if (!aligned16(L.k) || !aligned16(L.v)) return false;
    for (int q = 0; q < 3; ++q)
      if ((L.k_stride[q] * esize) % 16 || (L.v_stride[q] * esize) % 16) return false;
  }
  return true;
}

int resolve_plan(const gkv_plan* pp, int64_t S, bool quantize, const gkv_layer_in* layers, int n_layers,
                 bool outputs_aligned, Resolved& r) {
  if (!pp) return fail(GKV_ERR_INVALID, "plan is NULL");
  const gkv_plan& p = *pp;
  if (p.batch < 1 || p.head_dim < 1 || p.seq_len < 1) return fail(GKV_ERR_INVALID, "batch, head_dim, seq_len >= 1");
  if (p.dtype < GKV_F32 || p.dtype > GKV_BF16) return fail(GKV_ERR_INVALID, "bad dtype");
  if (p.n_retained < 0 || p.n_standard < 0 || p.n_cold < 0 ||
      (int64_t)p.n_retained + p.n_standard + p.n_cold != p.seq_len)
    return fail(GKV_ERR_INVALID, "tier lengths must be >= 0 and sum to seq_len");
  if ((p.n_retained && !p.idx_retained) || (p.n_standard && !p.idx_standard) || (p.n_cold && !p.idx_cold))
    return fail(GKV_ERR_INVALID, "missing index list");
  if (p.n_retained && (!p.retained_k || !p.retained_v)) return fail(GKV_ERR_INVALID, "missing retained storage");
  r.n[0] = p.n_retained;
  r.n[1] = p.n_standard;
  r.n[2] = p.n_cold;
  const int D = p.head_dim;
  const int esize = elem_size(p.dtype);
  bool any_rot = false;
  for (int i = 0; i < 4; ++i) {
    r.t[i] = TensorDesc{};
    const int n = r.n[kTierOf[i]];
    if (n == 0) continue;
    const int st = resolve_tensor(p, i, n, r.t[i]);
    if (st != GKV_OK) return st;
    any_rot |= r.t[i].rotation != 0;
    if (quantize && n_layers > 1 && r.t[i].packed && (r.t[i].elems_slice * r.t[i].sbits) % 8)
      return fail(GKV_ERR_INVALID, "codes of one slice are not whole bytes: call one layer at a time");
  }
  if (any_rot && !(p.hadamard_divisor > 0.f)) return fail(GKV_ERR_INVALID, "hadamard_divisor must be > 0");

  // tile routing
  const bool geom_ok = (D * esize) % 16 == 0 && tile_instantiated(esize, D, 64) && outputs_aligned &&
                       (!quantize || layers_aligned(layers, n_layers, esize));
  const bool ret_ok = p.n_retained == 0 || (aligned16(p.retained_k) && aligned16(p.retained_v));
  int tt = 64;
  bool want[3] = {false, false, false};
  for (int tier = 1; tier <= 2; ++tier) {
    if (!geom_ok || r.n[tier] == 0) continue;
    want[tier] = true;
  }
  r.tt = tt;
  for (int tier = 1; tier <= 2; ++tier) {
    bool ok = want[tier];
    for (int i = 0; i < 4 && ok; ++i)
      if (kTierOf[i] == tier) ok = tensor_fast(r.t[i], esize, D, tt, quantize);
    r.fast[tier] = ok;
  }
  r.fast[0] = geom_ok && ret_ok && p.n_retained > 0;

  // workspace of the general quantize path
  size_t off = 0;
  for (int i = 0; i < 4; ++i) {
    r.ws_scale[i] = r.ws_rot[i] = 0;
    const int tier = kTierOf[i];
    if (!quantize || r.n[tier] == 0 || r.fast[tier]) continue;
    r.ws_scale[i] = off;
    off = align256(off + (size_t)S * r.t[i].groups_slice * sizeof(float));
    if (r.t[i].rotation) {
      r.ws_rot[i] = off;
      off = align256(off + (size_t)S * r.t[i].n * D * esize);
    }
  }
  r.ws_bytes = off;
  return GKV_OK;
}

int64_t total_slices(const gkv_plan& p, const gkv_layer_in* layers, int n_layers) {
  int64_t s = 0;
  for (int l = 0; l < n_layers; ++l) s += (int64_t)p.batch * layers[l].heads;
  return s;
}

}  // namespace
}  // namespace gkv

using namespace gkv;

extern "C" {

int32_t gkv_abi_version(void) { return GKV_ABI_VERSION; }

const char* gkv_last_error(void) { return g_last_error.c_str(); }

int32_t gkv_device_error(int32_t* code) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int v = 0;
  if ((e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int))) != cudaSuccess)
    return cuda_fail(e, "reading the device error word");
  const int zero = 0;
  if ((e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int))) != cudaSuccess)
    return cuda_fail(e, "clearing the device error word");
  if (code) *code = v;
  return GKV_OK;
}

size_t gkv_select_workspace_bytes(int32_t seq_len) { return seq_len > 0 ? select_workspace(seq_len) : 0; }

int32_t gkv_select_tiers(const float* scores, const float* outlier_scores, const gkv_select_policy* pol,
                         int32_t* idx_retained, int32_t* idx_standard, int32_t* idx_cold, void* workspace,
                         size_t workspace_bytes, gkv_stream_t stream) {
  if (!pol) return fail(GKV_ERR_INVALID, "policy is NULL");
  const gkv_select_policy& p = *pol;
  const int T = p.seq_len;
  if (T < 1) return fail(GKV_ERR_INVALID, "seq_len must be >= 1");
  if (p.sink < 0 || p.sink > T || p.tail < 0 || p.tail > T || p.keep_protect < 0 || p.keep_outlier < 0 ||
      p.keep_cold < 0)
    return fail(GKV_ERR_INVALID, "sink/tail/keep counts out of range");
  if (p.n_retained < 0 || p.n_standard < 0 || p.n_cold < 0 ||
      (int64_t)p.n_retained + p.n_standard + p.n_cold != T)
    return fail(GKV_ERR_INVALID, "tier lengths must sum to seq_len");
  if ((p.keep_protect || p.keep_cold) && !scores) return fail(GKV_ERR_INVALID, "scores required");
  if (p.keep_outlier && !outlier_scores) return fail(GKV_ERR_INVALID, "outlier scores required");
  if ((p.n_retained && !idx_retained) || (p.n_standard && !idx_standard) || (p.n_cold && !idx_cold))
    return fail(GKV_ERR_INVALID, "missing index list output");
  if (!workspace || workspace_bytes < select_workspace(T))
    return fail(GKV_ERR_WORKSPACE, "selection workspace too small");
  cudaError_t e = launch_select(scores, outlier_scores, p, idx_retained, idx_standard, idx_cold,
                                static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GKV_OK : cuda_fail(e, "select kernel launch");
}

int32_t gkv_mean_scores(const float* scores, int32_t rows, int32_t cols, int32_t axis, int32_t last_block,
                        float* out, gkv_stream_t stream) {
  if (!scores || !out) return fail(GKV_ERR_INVALID, "NULL argument");
  if (rows < 1 || cols < 1) return fail(GKV_ERR_INVALID, "rows and cols must be >= 1");
  if (axis != 0 && axis != 1) return fail(GKV_ERR_INVALID, "axis must be 0 or 1");
  if (axis == 0 && (last_block < 0 || last_block >= cols || last_block % 32))
    return fail(GKV_ERR_INVALID, "last_block must be a multiple of 32 in [0, cols)");
  cudaError_t e = launch_mean_scores(scores, rows, cols, axis, axis == 0 ? last_block : 0, out,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GKV_OK : cuda_fail(e, "score mean kernel launch");
}

int32_t gkv_outlier_scores(const gkv_layer_in* layer, int32_t batch, int32_t seq_len, int32_t head_dim,
                           int32_t dtype, float* out, gkv_stream_t stream) {
  if (!layer || !layer->k || !layer->v || !out) return fail(GKV_ERR_INVALID, "NULL argument");
  if (batch < 1 || seq_len < 1 || head_dim < 1 || layer->heads < 1) return fail(GKV_ERR_INVALID, "bad geometry");
  if (dtype < GKV_F32 || dtype > GKV_BF16) return fail(GKV_ERR_INVALID, "bad dtype");
  cudaError_t e = launch_outlier(*layer, batch, seq_len, head_dim, dtype, out, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GKV_OK : cuda_fail(e, "outlier kernel launch");
}

size_t gkv_quantize_workspace_bytes(const gkv_plan* plan, const gkv_layer_in* layers, int32_t n_layers) {
  if (!plan || !layers || n_layers < 1) return 0;
  Resolved r;
  if (resolve_plan(plan, total_slices(*plan, layers, n_layers), true, layers, n_layers, true, r) != GKV_OK) return 0;
  return r.ws_bytes;
}

int32_t gkv_quantize(const gkv_plan* plan, const gkv_layer_in* layers, int32_t n_layers, void* workspace,
                     size_t workspace_bytes, gkv_stream_t stream) {
  if (!plan || !layers || n_layers < 1) return fail(GKV_ERR_INVALID, "plan/layers missing");
  for (int l = 0; l < n_layers; ++l)
    if (!layers[l].k || !layers[l].v || layers[l].heads < 1) return fail(GKV_ERR_INVALID, "bad layer input");
  const int64_t S_total = total_slices(*plan, layers, n_layers);
  if (S_total > (int64_t)1 << 30) return fail(GKV_ERR_TOO_LARGE, "too many slices");
  Resolved r;
  int st = resolve_plan(plan, S_total, true, layers, n_layers, true, r);
  if (st != GKV_OK) return st;
  if (r.ws_bytes && (!workspace || workspace_bytes < r.ws_bytes))
    return fail(GKV_ERR_WORKSPACE, "workspace too small: need " + std::to_string(r.ws_bytes) + " bytes");
  for (int i = 0; i < 4; ++i) {
    if (r.ws_bytes == 0 || r.fast[kTierOf[i]] || r.n[kTierOf[i]] == 0) continue;
    r.t[i].scale32 = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + r.ws_scale[i]);
    if (r.t[i].rotation) r.t[i].rot = static_cast<uint8_t*>(workspace) + r.ws_rot[i];
  }
  const gkv_plan& p = *plan;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  QuantParams q;
  q.B = p.batch;
  q.T = p.seq_len;
  q.D = p.head_dim;
  q.idx[0] = p.idx_retained;
  q.idx[1] = p.idx_standard;
  q.idx[2] = p.idx_cold;
  for (int k = 0; k < 3; ++k) q.n_tier[k] = r.n[k];
  for (int i = 0; i < 4; ++i) q.t[i] = r.t[i];
  q.ret_k = p.retained_k;
  q.ret_v = p.retained_v;
  q.had_div = p.hadamard_divisor;
  q.had_inv = p.hadamard_divisor > 0.f ? 1.0f / p.hadamard_divisor : 0.f;
  // the fused quotient y * (1 / div) + correction is proven exact (|quotient| >=
  // 2^-100) for fp32(sqrt(D)) at the tile head dims 64 (a power of two) and 128
  q.had_fused = (p.head_dim == 64 || p.head_dim == 128) &&
                p.hadamard_divisor == (float)std::sqrt((double)p.head_dim);
  q.tt = r.tt;
  q.tiles[0] = r.fast[0] ? (int)ceil_div(r.n[0], kRetTile) : 0;
  for (int k = 1; k <= 2; ++k) q.tiles[k] = r.fast[k] ? (int)ceil_div(r.n[k], r.tt) : 0;
  q.tiles_slice = q.tiles[0] + q.tiles[1] + q.tiles[2];
  q.tile_div = make_fastdiv((uint32_t)(q.tiles_slice > 0 ? q.tiles_slice : 1));
  int64_t slice0 = 0;
  for (int l0 = 0; l0 < n_layers; l0 += kMaxLayers) {
    const int nl = n_layers - l0 < kMaxLayers ? n_layers - l0 : kMaxLayers;
    int S = 0;
    for (int l = 0; l < nl; ++l) {
      const gkv_layer_in& L = layers[l0 + l];
      LayerDesc& d = q.layers[l];
      d.k = L.k;
      d.v = L.v;
      for (int c = 0; c < 3; ++c) { d.ks[c] = L.k_stride[c]; d.vs[c] = L.v_stride[c]; }
      d.heads = L.heads;
      d.slice_begin = S;
      S += p.batch * L.heads;
    }
    q.n_layers = nl;
    q.S = S;
    q.slice_offset = (int)slice0;
    bool uniform = true;
    for (int l = 1; l < nl; ++l) uniform &= q.layers[l].heads == q.layers[0].heads;
    q.layer_div = uniform ? make_fastdiv((uint32_t)(p.batch * q.layers[0].heads)) : FastDiv{0u, 0u, 0, 0};
    q.head_div = make_fastdiv((uint32_t)q.layers[0].heads);
    cudaError_t e = cudaSuccess;
    if (q.tiles_slice > 0) {
      SideStreamCall side(s, (int64_t)q.S * q.tiles_slice >= kSideMinTiles);
      if ((e = side.error()) != cudaSuccess) return cuda_fail(e, "side stream");
      e = launch_quantize_tiles(q, p.dtype, s, side.side());
      const cudaError_t ej = side.join();
      if (e != cudaSuccess) return cuda_fail(e, "quantize tile kernel");
      if (ej != cudaSuccess) return cuda_fail(ej, "side stream join");
    }
    if (!r.fast[0] && r.n[0] > 0 && (e = launch_retained_general(q, p.dtype, s)) != cudaSuccess)
      return cuda_fail(e, "retained copy kernel");
    for (int i = 0; i < 4; ++i) {
      const int tier = kTierOf[i];
      if (r.n[tier] == 0 || r.fast[tier]) continue;
      if ((e = launch_quantize_general(q, p.dtype, i, tier, s)) != cudaSuccess)
        return cuda_fail(e, "general quantize kernels");
    }
    slice0 += S;
  }
  return GKV_OK;
}

size_t gkv_dequantize_workspace_bytes(const gkv_plan* plan, int32_t n_slices) {
  (void)plan;
  (void)n_slices;
  return 0;
}

int32_t gkv_dequantize(const gkv_plan* plan, int32_t n_slices, void* k_out, void* v_out, void* workspace,
                       size_t workspace_bytes, gkv_stream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (!plan || !k_out || !v_out || n_slices < 1) return fail(GKV_ERR_INVALID, "plan/outputs missing");
  Resolved r;
  // the tile kernels store 16-byte vectors: every output slice must start 16-byte aligned
  const int64_t out_T = plan && plan->out_seq_stride ? plan->out_seq_stride : (plan ? plan->seq_len : 0);
  const bool out_aligned = aligned16(k_out) && aligned16(v_out) && plan &&
                           (out_T * plan->head_dim * elem_size(plan->dtype)) % 16 == 0;
  int st = resolve_plan(plan, n_slices, false, nullptr, 0, out_aligned, r);
  if (st != GKV_OK) return st;
  const gkv_plan& p = *plan;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.out_seq_stride != 0 && p.out_seq_stride < p.seq_len)
    return fail(GKV_ERR_INVALID, "out_seq_stride must be 0 or >= seq_len");
  DequantParams q;
  q.T = p.seq_len;
  q.D = p.head_dim;
  q.S = n_slices;
  q.out_T = p.out_seq_stride ? p.out_seq_stride : p.seq_len;
  q.idx[0] = p.idx_retained;
  q.idx[1] = p.idx_standard;
  q.idx[2] = p.idx_cold;
  for (int k = 0; k < 3; ++k) q.n_tier[k] = r.n[k];
  for (int i = 0; i < 4; ++i) q.t[i] = r.t[i];
  q.ret_k = p.retained_k;
  q.ret_v = p.retained_v;
  q.out_k = k_out;
  q.out_v = v_out;
  q.had_div = p.hadamard_divisor;
  q.had_inv = p.hadamard_divisor > 0.f ? 1.0f / p.hadamard_divisor : 0.f;
  q.tt = r.tt;
  q.tiles[0] = r.fast[0] ? (int)ceil_div(r.n[0], kRetTile) : 0;
  for (int k = 1; k <= 2; ++k) q.tiles[k] = r.fast[k] ? (int)ceil_div(r.n[k], r.tt) : 0;
  q.tiles_slice = q.tiles[0] + q.tiles[1] + q.tiles[2];
  q.tile_div = make_fastdiv((uint32_t)(q.tiles_slice > 0 ? q.tiles_slice : 1));
  q.had_fused = (p.head_dim == 64 || p.head_dim == 128) &&
                p.hadamard_divisor == (float)std::sqrt((double)p.head_dim);
  cudaError_t e;
  if (q.tiles_slice > 0) {
    SideStreamCall side(s, (int64_t)q.S * q.tiles_slice >= kSideMinTiles);
    if ((e = side.error()) != cudaSuccess) return cuda_fail(e, "side stream");
    e = launch_dequantize_tiles(q, p.dtype, s, side.side());
    const cudaError_t ej = side.join();
    if (e != cudaSuccess) return cuda_fail(e, "dequantize tile kernel");
    if (ej != cudaSuccess) return cuda_fail(ej, "side stream join");
  }
  if (!r.fast[0] && r.n[0] > 0 && (e = launch_dequantize_retained_general(q, p.dtype, s)) != cudaSuccess)
    return cuda_fail(e, "retained scatter kernel");
  for (int tier = 1; tier <= 2; ++tier) {
    if (r.n[tier] == 0 || r.fast[tier]) continue;
    if ((e = launch_dequantize_general(q, p.dtype, tier, s)) != cudaSuccess)
      return cuda_fail(e, "general dequantize kernel");
  }
  return GKV_OK;
}

namespace {

// Tiles per slice of a dequant / attention call (retained, standard, cold).
void tile_counts(const Resolved& r, int* tiles) {
  tiles[0] = r.fast[0] ? (int)ceil_div(r.n[0], kRetTile) : 0;
  for (int k = 1; k <= 2; ++k) tiles[k] = r.fast[k] ? (int)ceil_div(r.n[k], r.tt) : 0;
}

// The attention kernels cover layers whose every non-empty tier takes the tile
// path, with keys grouped along tokens (not rotated) and values along channels.
int resolve_attention(const gkv_plan* plan, int32_t n_slices, int32_t n_queries, Resolved& r) {
  if (!plan) return fail(GKV_ERR_INVALID, "plan is NULL");
  if (n_slices < 1 || n_queries < 1) return fail(GKV_ERR_INVALID, "n_slices and n_queries must be >= 1");
  if (n_queries > kAttnMaxQueries)
    return fail(GKV_ERR_TOO_LARGE, "at most " + std::to_string(kAttnMaxQueries) + " queries per slice");
  const int st = resolve_plan(plan, n_slices, false, nullptr, 0, true, r);
  if (st != GKV_OK) return st;
  const gkv_plan& p = *plan;
  if (p.head_dim != 64 && p.head_dim != 128) return fail(GKV_ERR_UNSUPPORTED, "attention: head_dim must be 64 or 128");
  for (int tier = 0; tier <= 2; ++tier)
    if (r.n[tier] > 0 && !r.fast[tier]) return fail(GKV_ERR_UNSUPPORTED, "attention: a tier outside the tile path");
  for (int tier = 1; tier <= 2; ++tier) {
    if (r.n[tier] == 0) continue;
    const TensorDesc& k = r.t[tier == 1 ? GKV_STD_K : GKV_COLD_K];
    const TensorDesc& v = r.t[tier == 1 ? GKV_STD_V : GKV_COLD_V];
    if (k.axis != GKV_AXIS_TOKEN || k.rotation || v.axis != GKV_AXIS_CHANNEL)
      return fail(GKV_ERR_UNSUPPORTED, "attention: keys grouped along tokens and values along channels only");
  }
  return GKV_OK;
}

}  // namespace

// Softmax partials of every tile, then those of the first merge stage's groups.
static size_t attention_workspace(int n_slices, int tiles_slice, int n_queries, int head_dim) {
  const size_t entry = (size_t)n_queries * (head_dim + 2) * sizeof(float);
  return (size_t)n_slices * (tiles_slice + merge_groups(tiles_slice)) * entry;
}

size_t gkv_attention_workspace_bytes(const gkv_plan* plan, int32_t n_slices, int32_t n_queries) {
  Resolved r;
  if (resolve_attention(plan, n_slices, n_queries, r) != GKV_OK) return 0;
  int tiles[3];
  tile_counts(r, tiles);
  const int n = tiles[0] + tiles[1] + tiles[2];
  return attention_workspace(n_slices, n, n_queries, plan->head_dim);
}

int32_t gkv_attention(const gkv_plan* plan, int32_t n_slices, const float* queries, int32_t n_queries, float* out,
                      void* workspace, size_t workspace_bytes, gkv_stream_t stream) {
  if (!queries || !out) return fail(GKV_ERR_INVALID, "queries / out missing");
  Resolved r;
  int st = resolve_attention(plan, n_slices, n_queries, r);
  if (st != GKV_OK) return st;
  const gkv_plan& p = *plan;
  AttnParams a;
  DequantParams& q = a.d;
  q.T = p.seq_len;
  q.D = p.head_dim;
  q.S = n_slices;
  q.out_T = p.seq_len;
  q.idx[0] = p.idx_retained;
  q.idx[1] = p.idx_standard;
  q.idx[2] = p.idx_cold;
  for (int k = 0; k < 3; ++k) q.n_tier[k] = r.n[k];
  for (int i = 0; i < 4; ++i) q.t[i] = r.t[i];
  q.ret_k = p.retained_k;
  q.ret_v = p.retained_v;
  q.out_k = q.out_v = nullptr;
  q.had_div = p.hadamard_divisor;
  q.had_inv = p.hadamard_divisor > 0.f ? 1.0f / p.hadamard_divisor : 0.f;
  q.had_fused = (p.head_dim == 64 || p.head_dim == 128) &&
                p.hadamard_divisor == (float)std::sqrt((double)p.head_dim);
  q.tt = r.tt;
  tile_counts(r, q.tiles);
  q.tiles_slice = q.tiles[0] + q.tiles[1] + q.tiles[2];
  q.tile_div = make_fastdiv((uint32_t)(q.tiles_slice > 0 ? q.tiles_slice : 1));
  const size_t need = attention_workspace(n_slices, q.tiles_slice, n_queries, p.head_dim);
  if (!workspace || workspace_bytes < need)
    return fail(GKV_ERR_WORKSPACE, "attention workspace too small: need " + std::to_string(need) + " bytes");
  a.q = queries;
  a.Q = n_queries;
  a.inv_sqrt_d = (float)(1.0 / std::sqrt((double)p.head_dim));
  a.part = static_cast<float*>(workspace);
  a.part2 = a.part + (size_t)n_slices * q.tiles_slice * n_queries * (p.head_dim + 2);
  a.out = out;
  cudaError_t e = launch_attention(a, p.dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GKV_OK : cuda_fail(e, "attention kernels");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Tier selection without any device allocation.
//
// The selection kernel needs one byte of tier state per token.  gkv_select_tiers
// takes that scratch from the caller; this variant uses a fixed array owned by
// the library instead, for callers that cannot allocate device memory when they
// select (for instance an engine that has handed all free device memory to its
// own pool, or a latency-critical path where cudaMalloc's implicit device-wide
// synchronisation is not acceptable).
// ---------------------------------------------------------------------------

namespace gkv {
namespace {

constexpr int kStaticSelectMaxTokens = GKV_STATIC_SELECT_MAX_TOKENS;
constexpr int kMaxDevices = 64;

// Selection workspace for kStaticSelectMaxTokens tokens (13 MiB and 256 bytes:
// tier bytes plus the three 4-byte tables of the exact tie path).  Every GPU that loads this
// library holds it until the process exits.  In host code `g_select_scratch`
// only names a host-side handle of the symbol; the device address comes from
// cudaGetSymbolAddress below.
constexpr size_t kStaticSelectBytes = select_workspace(kStaticSelectMaxTokens);
static __device__ __align__(256) uint8_t g_select_scratch[kStaticSelectBytes];

std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of the scratch on the current device, looked up once per device.
int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(GKV_ERR_UNSUPPORTED, "device ordinal beyond 63");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_address[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_select_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(selection scratch)");
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
  return GKV_OK;
}

}  // namespace
}  // namespace gkv

extern "C" int32_t gkv_select_tiers_static(const float* scores, const float* outlier_scores,
                                           const gkv_select_policy* policy, int32_t* idx_retained,
                                           int32_t* idx_standard, int32_t* idx_cold, gkv_stream_t stream) {
  if (!policy) return fail(GKV_ERR_INVALID, "policy is NULL");
  if (policy->seq_len > kStaticSelectMaxTokens)
    return fail(GKV_ERR_TOO_LARGE, "seq_len " + std::to_string(policy->seq_len) +
                                       " exceeds the library's static selection scratch of " +
                                       std::to_string(kStaticSelectMaxTokens) + " tokens");
  void* scratch = nullptr;
  const int st = static_scratch_address(&scratch);
  if (st != GKV_OK) return st;
  // the kernel writes the tier byte of every token before reading it, so the
  // previous call's contents need no clearing
  return gkv_select_tiers(scores, outlier_scores, policy, idx_retained, idx_standard, idx_cold, scratch,
                          kStaticSelectBytes, stream);
}
