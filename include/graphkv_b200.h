/*
 * graphkv_b200.h -- C ABI of the B200 (sm_100a) GraphKV cache-compression kernels.
 *
 * The reference implements this path as PyTorch ATen calls in
 * src/graphkv/core.py; each entry point below names the reference function(s)
 * whose data path it replaces.  The host side (graphkv_b200/*.py) mirrors the
 * reference's Python API and calls these entry points through ctypes.
 *
 * Conventions
 *  - All pointers are device pointers unless stated otherwise; sizes are in
 *    elements unless stated otherwise.
 *  - `stream` is a cudaStream_t passed as void*; all work is ordered on it and
 *    every entry point returns without synchronising.  (gkv_quantize and
 *    gkv_dequantize may run their rotated-tier kernels on a library-owned
 *    stream of the same GPU, started after the work already on `stream` and
 *    joined back into `stream` before the call returns, so later work on
 *    `stream` sees their results.  The first such call on a device creates that
 *    stream and its two events; make it before any stream capture.)
 *  - Return value: GKV_OK (0) or a negative gkv_status; gkv_last_error()
 *    returns a message for the calling thread's last failure.
 *  - Kernels record problems they find in the data (an index list entry outside
 *    [0, T): 3; selection counts that differ from the plan: 2) in a per-device
 *    error word and carry on without the faulty access; gkv_device_error()
 *    reads and clears that word (it synchronises the device).
 *
 * Terms
 *  - slice: one (layer, batch row, kv-head) matrix [T, D] of keys or values.
 *    A call covers S slices, ordered layer-major, then batch row, then head.
 *  - tiers: retained (kept in the input dtype), standard (quantized with the
 *    base bits) and cold (low-priority, quantized with the low-priority bits),
 *    given by three ascending lists of token positions.
 */
#ifndef GRAPHKV_B200_H
#define GRAPHKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GKV_ABI_VERSION 1

typedef void* gkv_stream_t; /* cudaStream_t */

typedef enum {
  GKV_OK = 0,
  GKV_ERR_INVALID = -1,     /* bad argument (maps to ValueError on the Python side) */
  GKV_ERR_UNSUPPORTED = -2, /* valid but unsupported combination */
  GKV_ERR_CUDA = -3,        /* a CUDA runtime call failed */
  GKV_ERR_WORKSPACE = -4,   /* workspace missing or too small */
  GKV_ERR_TOO_LARGE = -5    /* size beyond a stated maximum */
} gkv_status;

typedef enum { GKV_F32 = 0, GKV_F16 = 1, GKV_BF16 = 2 } gkv_dtype;
typedef enum { GKV_SYMMETRIC = 0, GKV_AFFINE = 1 } gkv_quantizer;
typedef enum { GKV_AXIS_TOKEN = 0, GKV_AXIS_CHANNEL = 1 } gkv_axis;
typedef enum { GKV_ROT_NONE = 0, GKV_ROT_HADAMARD = 1 } gkv_rotation;
typedef enum { GKV_STD_K = 0, GKV_STD_V = 1, GKV_COLD_K = 2, GKV_COLD_V = 3 } gkv_tensor_slot;

/* How one of the four compressed tensors is quantized (core.py:848-910). */
typedef struct gkv_tensor_spec {
  int32_t bits;        /* 2, 4 or 8 */
  int32_t quantizer;   /* gkv_quantizer */
  int32_t axis;        /* gkv_axis: GKV_AXIS_TOKEN groups consecutive tier tokens of one
                          channel (codes stored [D, n_pad] per slice); GKV_AXIS_CHANNEL
                          groups consecutive channels of one token ([n, D_pad] per slice) */
  int32_t group_size;  /* effective group size = min(configured group_size, axis length) */
  int32_t rotation;    /* gkv_rotation: Hadamard over head_dim before quantizing */
  int32_t packed;      /* 1: 8/bits codes per byte, element 0 in the low bits, code - qmin
                          stored (core.py:979-990); 0: one int8 (symmetric) / uint8 (affine)
                          code per byte */
  int32_t scale_dtype; /* gkv_dtype of the stored scales */
  int32_t reserved;
} gkv_tensor_spec;

/* Everything about one call except the input K/V pointers.
 * For gkv_quantize the storage pointers are outputs, for gkv_dequantize inputs.
 * Each storage field is ONE region covering all S slices of the call, in slice
 * order; the per-slice extents follow from the geometry and the specs:
 *   retained rows         n_retained * D elements of `dtype`
 *   token-axis tensor     codes for D * n_pad elements, D * n_pad / group_size scales
 *   channel-axis tensor   codes for n * D_pad elements, n * D_pad / group_size scales
 * with n the tier length, n_pad = ceil(n / gs) * gs, D_pad = ceil(D / gs) * gs.
 * Packed codes form one little-end-first stream per layer (core.py:979-990);
 * when a slice's code count is not a whole number of bytes a call must cover
 * exactly one layer. */
typedef struct gkv_plan {
  int32_t batch;       /* B */
  int32_t head_dim;    /* D */
  int32_t seq_len;     /* T */
  int32_t dtype;       /* gkv_dtype of K/V and of the retained rows */
  int32_t n_retained;  /* R  */
  int32_t n_standard;  /* Tc */
  int32_t n_cold;      /* Tl */
  int32_t out_seq_stride; /* gkv_dequantize: tokens between two output slices (0: seq_len) --
                             lets a dequantize write into a longer [S, stride, D] buffer */
  const int32_t* idx_retained; /* [R]  ascending token positions */
  const int32_t* idx_standard; /* [Tc] */
  const int32_t* idx_cold;     /* [Tl] */
  gkv_tensor_spec spec[4];     /* indexed by gkv_tensor_slot */
  float hadamard_divisor;      /* fp32(sqrt(D)) -- the reference divides by it (core.py:956) */
  int32_t reserved1;
  void* retained_k;            /* [S, R, D] */
  void* retained_v;
  uint8_t* codes[4];
  void* scales[4];
  uint8_t* zero_points[4];     /* uint8 per group; NULL for symmetric tensors */
} gkv_plan;

/* One layer's input keys/values [B, H, T, D]; head_dim must be contiguous. */
typedef struct gkv_layer_in {
  const void* k;
  const void* v;
  int64_t k_stride[3];  /* element strides of the batch, head and token dims */
  int64_t v_stride[3];
  int32_t heads;        /* H of this layer */
  int32_t reserved;
} gkv_layer_in;

/* Retention policy of one selection, resolved on the host from the config and
 * T (all counts are known before any kernel runs). */
typedef struct gkv_select_policy {
  int32_t seq_len;          /* T */
  int32_t sink;             /* tokens [0, sink) retained */
  int32_t tail;             /* tokens [T - tail, T) retained */
  int32_t keep_protect;     /* largest importance scores retained among the rest */
  int32_t keep_outlier;     /* largest outlier scores retained among the rest after that */
  int32_t keep_cold;        /* smallest importance scores moved to the cold tier */
  int32_t n_retained;       /* expected list lengths (checked on the device) */
  int32_t n_standard;
  int32_t n_cold;
  int32_t reserved;
} gkv_select_policy;

int32_t gkv_abi_version(void);
const char* gkv_last_error(void);

/* Reads and clears the per-device error word of the current device (0 = none).
 * Synchronises the device. */
int32_t gkv_device_error(int32_t* code);

/* Tier selection: sink/tail retention, top-k importance protection, top-k
 * outlier protection and bottom-k cold tier, then the three ascending index
 * lists.  Replaces build_retention_mask (core.py:595-644),
 * _apply_score_retention (core.py:1034-1048), the cold-tier topk
 * (core.py:685-712) and the index lists (core.py:716-719).  Among equal scores
 * at a selection boundary the tokens are those torch.topk picks on the CPU
 * (the order of libstdc++'s partial_sort / nth_element over the candidates).
 * scores / outlier_scores: fp32 [T] (outlier_scores may be NULL when
 * keep_outlier == 0).  workspace: gkv_select_workspace_bytes(T) bytes
 * (13 bytes per token, 256-byte aligned regions). */
size_t gkv_select_workspace_bytes(int32_t seq_len);
int32_t gkv_select_tiers(const float* scores, const float* outlier_scores, const gkv_select_policy* policy,
                         int32_t* idx_retained, int32_t* idx_standard, int32_t* idx_cold,
                         void* workspace, size_t workspace_bytes, gkv_stream_t stream);

/* Same selection as gkv_select_tiers, but the library supplies the scratch:
 * no workspace argument, and nothing is allocated by the caller or by the
 * library during the call.  This entry point has no counterpart in the
 * reference; it exists for callers that cannot allocate device memory when they
 * select -- e.g. an engine that has given all free device memory to its own
 * pool, or a latency-critical path that cannot afford cudaMalloc's implicit
 * device-wide synchronisation.
 *  - Limit: seq_len <= GKV_STATIC_SELECT_MAX_TOKENS; larger sizes return
 *    GKV_ERR_TOO_LARGE without launching anything.
 *  - The scratch is a 13 MiB (+256 B) device array inside the library (the selection
 *    workspace of GKV_STATIC_SELECT_MAX_TOKENS tokens); every GPU that loads
 *    the library keeps it until the process exits.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.
 *  - Each GPU has its own copy of the array, shared by every call on that
 *    GPU: calls on one GPU whose kernels can overlap (different streams, or
 *    several host threads) race and must be ordered by the caller; calls on
 *    different GPUs do not interact.  No clearing is needed between calls: the
 *    kernel writes every token's tier byte before reading it. */
#define GKV_STATIC_SELECT_MAX_TOKENS 1048576
int32_t gkv_select_tiers_static(const float* scores, const float* outlier_scores, const gkv_select_policy* policy,
                                int32_t* idx_retained, int32_t* idx_standard, int32_t* idx_cold,
                                gkv_stream_t stream);

/* Mean of fp32 scores [rows, cols] (contiguous) over axis 0 (-> [cols]) or
 * axis 1 (-> [rows]).  Replaces the averaging of multi-dimensional importance
 * scores in _normalize_token_scores (core.py:1027-1030: reshape(-1, T).mean(0)
 * and reshape(T, -1).mean(1)), bit-identical to torch's CPU mean: the sums
 * follow the fp32 addition order of ATen's CPU cascade sum, then one division
 * by the count.  last_block (axis 0 only): first column of the last per-thread
 * column block of that CPU reduction, a multiple of 32 that depends on the
 * thread count (0 for a single-threaded reduction); the Python layer derives
 * it from torch.get_num_threads(). */
int32_t gkv_mean_scores(const float* scores, int32_t rows, int32_t cols, int32_t axis, int32_t last_block,
                        float* out, gkv_stream_t stream);

/* Per-token outlier score mean(K^2) + mean(V^2) over (batch, head, head_dim)
 * for one layer, fp32 [T].  Replaces _kv_outlier_scores (core.py:1051-1054);
 * sums are accumulated in fp64 and rounded once. */
int32_t gkv_outlier_scores(const gkv_layer_in* layer, int32_t batch, int32_t seq_len, int32_t head_dim,
                           int32_t dtype, float* out, gkv_stream_t stream);

/* Quantize + pack every tier of every slice of n_layers layers in one launch.
 * Replaces, per layer, the data path of quantize_kv_layer (core.py:647-772):
 * the index_select gathers (core.py:721-722, 729-730, 738-739),
 * _quantize_tensor (core.py:848-910), _hadamard_last_dim (core.py:945-956)
 * and _pack_lowbit (core.py:979-990); over layers it replaces the loop of
 * QuantizedKvCache.from_past_key_values (core.py:355-369). */
size_t gkv_quantize_workspace_bytes(const gkv_plan* plan, const gkv_layer_in* layers, int32_t n_layers);
int32_t gkv_quantize(const gkv_plan* plan, const gkv_layer_in* layers, int32_t n_layers,
                     void* workspace, size_t workspace_bytes, gkv_stream_t stream);

/* Unpack + dequantize every tier of n_slices slices and scatter the rows, with
 * the retained rows, into k_out / v_out ([S, T, D], or [S, out_seq_stride, D]
 * whose first T rows of each slice are written, dtype of the plan); every
 * output row is written exactly once.  Replaces
 * QuantizedKvLayer.dequantize (core.py:265-307), QuantizedTensor.dequantize
 * (core.py:153-173) and _unpack_lowbit (core.py:993-1007); over layers,
 * QuantizedKvCache.dequantize (core.py:371-372). */
size_t gkv_dequantize_workspace_bytes(const gkv_plan* plan, int32_t n_slices);
int32_t gkv_dequantize(const gkv_plan* plan, int32_t n_slices, void* k_out, void* v_out,
                       void* workspace, size_t workspace_bytes, gkv_stream_t stream);

/* Attention of n_queries fp32 queries per slice ([S, n_queries, D], S =
 * batch * kv-heads) over a compressed layer, reading the packed codes directly:
 * out[s, i, :] = softmax(q_i k^T / sqrt(D)) v over the slice's dequantized keys
 * and values, without writing them out.  The reference computes this as
 * attention_from_kv over QuantizedKvLayer.dequantize() (core.py:800-820,
 * 265-307); the rows attended over are bit-identical to the dequantized
 * cache's, only the fp32 summation order differs.  Supported: head_dim 64 or
 * 128, every tier on the tile path, keys grouped along tokens (not rotated),
 * values along channels; otherwise GKV_ERR_UNSUPPORTED.  At most 16 queries.
 * workspace: gkv_attention_workspace_bytes(...) bytes (softmax partials per tile and per merge group). */
size_t gkv_attention_workspace_bytes(const gkv_plan* plan, int32_t n_slices, int32_t n_queries);
int32_t gkv_attention(const gkv_plan* plan, int32_t n_slices, const float* queries, int32_t n_queries, float* out,
                      void* workspace, size_t workspace_bytes, gkv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GRAPHKV_B200_H */
