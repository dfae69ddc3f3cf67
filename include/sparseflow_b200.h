/*
 * sparseflow_b200.h -- C ABI of the B200 (sm_100a) spike-sparse convolution path.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and a CUDA stream (passed as void*,
 *     a cudaStream_t; NULL means the legacy default stream);
 *   - only enqueues work on that stream (no host synchronisation, no device
 *     allocation) and returns a status code; it never throws;
 *   - has no CPU fallback: a configuration the kernels do not cover returns
 *     SF_ERR_UNSUPPORTED and the caller decides what to do.
 *
 * Reference interfaces replaced (paths inside hpcyhr/SparseFlow):
 *   sf_prescan2d          Kernels/_prescan_common.py:231-306 (_build_rf_prescan_metadata_impl,
 *                         build_rf_prescan_metadata) as called from
 *                         Kernels/conv2d.py:158-206 (_build_two_stage_metadata), fused with
 *                         Kernels/conv2d.py:113-123 (_build_active_tile_ids).
 *   sf_pack_weights       Ops/sparse_conv2d.py:339-350 (_get_w_cl weight repack).
 *   sf_sparse_conv2d      Kernels/conv2d.py:893-1178 (sparse_conv2d_forward: the
 *                         sparse_conv3x3s1/s2 and conv1x1 NHWC kernels, :236-886).
 *   sf_fused_conv_lif     Kernels/fused_conv_lif.py:310-484 (sparse_fused_conv_lif_forward)
 *                         with the LIF semantics of Ops/sparse_fused_conv_lif.py:271-293,
 *                         run over all T steps in one launch; optionally also writes the
 *                         next layer's event masks.
 *   sf_sparse_conv2d_from_masks, sf_event_masks_bytes
 *                         no reference counterpart: the consumer side of those masks.
 *   sf_lif_multistep      the multi-step LIFNode that follows a BN in spikingjelly-style
 *                         models (Ops/sparse_fused_conv_lif.py:271-293 applied over T;
 *                         spikingjelly LIFNode, step_mode 'm'), one launch for all steps.
 *   sf_lif_multistep_events  the same, also writing the next convolution's event masks.
 */
#ifndef SPARSEFLOW_B200_H
#define SPARSEFLOW_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SF_ABI_VERSION 1

typedef int32_t sf_status;
enum {
  SF_OK = 0,
  SF_ERR_INVALID_ARG = 1,   /* null pointer, non-positive size, inconsistent shape */
  SF_ERR_UNSUPPORTED = 2,   /* valid request outside what the kernels implement */
  SF_ERR_ALIGNMENT = 3,     /* a pointer is not 16-byte aligned */
  SF_ERR_WORKSPACE = 4,     /* workspace missing or too small */
  SF_ERR_CUDA = 5,          /* a CUDA runtime call failed (launch, attribute, ...) */
  SF_ERR_DEVICE_TIMEOUT = 6 /* reported by sf_prescan2d_status: a bounded device wait expired */
};

enum { SF_DTYPE_F32 = 0, SF_DTYPE_F16 = 1, SF_DTYPE_BF16 = 2 };
enum { SF_LAYOUT_NCHW = 0, SF_LAYOUT_NHWC = 1 };

/* Tile classes written by sf_prescan2d (Utils/sparse_helpers.py:28-30). */
enum { SF_TILE_ZERO = 0, SF_TILE_SPARSE = 1, SF_TILE_DENSEISH = 2 };

int32_t sf_abi_version(void);
const char* sf_status_string(sf_status s);

/* ------------------------------------------------------------------------ */
/* Stage 1: receptive-field prescan.                                         */
/* ------------------------------------------------------------------------ */
typedef struct sf_prescan_desc {
  int32_t n, c, h, w;          /* input dims; n folds T*B for 5-D inputs */
  int32_t h_out, w_out;        /* conv output dims */
  int32_t kernel, stride, padding;
  int32_t block_h, block_w;    /* output tile; GH = ceil(h_out/block_h) */
  int32_t group_size;          /* channels per group; ceil(c/group_size) <= 32 */
  double threshold;            /* compared as IEEE half, like the reference */
  int32_t dtype;               /* SF_DTYPE_* of x */
  int32_t layout;              /* SF_LAYOUT_* of x */
} sf_prescan_desc;

/* Bytes of caller-owned device workspace sf_prescan2d needs. The workspace
 * must be zero-filled once when first allocated; afterwards the kernel keeps it
 * consistent itself. One workspace serves one stream at a time. */
size_t sf_prescan2d_workspace_size(const sf_prescan_desc* d);

/* Writes, for the N*GH*GW tiles in (n, gh, gw) row-major order:
 *   ag_mask[t]     bit g set iff channel group g has |half(x)| > half(threshold)
 *                  somewhere in tile t's receptive field (NaN in that field
 *                  clears the bit, as max-pooling a NaN does in the reference);
 *   tile_class[t]  SF_TILE_ZERO / SPARSE / DENSEISH;
 *   active_ids     ascending ids of tiles with tile_class != ZERO;
 *   *active_count  their number.
 * active_ids / active_count may be NULL (then no compaction is done). */
sf_status sf_prescan2d(const void* x, const sf_prescan_desc* d,
                       int32_t* ag_mask, int32_t* tile_class,
                       int32_t* active_ids, int32_t* active_count,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Reads back (synchronously on `stream`) the device error word of a prescan
 * workspace: SF_OK or SF_ERR_DEVICE_TIMEOUT. Not for hot loops. */
sf_status sf_prescan2d_status(void* workspace, void* stream);

/* sf_prescan2d without a workspace argument, for callers that cannot allocate
 * device memory at the point they run the prescan (a host runtime that owns
 * every allocation, or a hot path where cudaMalloc would synchronise). No
 * counterpart in the reference: its prescan allocates through torch.
 * The look-back workspace is a static device array inside this library, sized
 * for at most SF_PRESCAN_STATIC_MAX_ROWS tile rows (n * ceil(h_out / block_h),
 * 256 KiB + 16 bytes per GPU, held until process exit); larger requests
 * return SF_ERR_WORKSPACE. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call before any
 * stream capture. Each call clears the counters it needs and allocates
 * nothing. All calls share the one array, so calls that may overlap on the
 * GPU (different streams, or several host threads) race and must be
 * serialised by the caller. */
#define SF_PRESCAN_STATIC_MAX_ROWS 32768
sf_status sf_prescan2d_static_ws(const void* x, const sf_prescan_desc* d,
                                 int32_t* ag_mask, int32_t* tile_class,
                                 int32_t* active_ids, int32_t* active_count, void* stream);

/* Error word of the most recent sf_prescan2d_static_ws call on the current
 * device (synchronous on `stream`): SF_OK, or SF_ERR_DEVICE_TIMEOUT when one
 * of that call's bounded look-back waits ran out (its active_ids are then not
 * valid). The next sf_prescan2d_static_ws call clears the word, so read it
 * before that. Not for hot loops. */
sf_status sf_prescan2d_static_ws_status(void* stream);

/* ------------------------------------------------------------------------ */
/* Stage 2: gather-style sparse convolution (deterministic, atomic-free).    */
/* ------------------------------------------------------------------------ */

/* Packed layout: [block][c_in][kernel*kernel][32][cpl], where block b holds
 * output channels b*32*cpl + j*32 + lane (j < cpl), zero padded past c_out;
 * cpl (1, 2 or 4) is the widest block whose weights fit in 160 KB, chosen by
 * the library from (c_out, c_in, kernel, dtype); element type w_dst_dtype
 * (F32 or BF16). Use sf_packed_weight_bytes for the size. */
size_t sf_packed_weight_bytes(int32_t c_out, int32_t c_in, int32_t kernel, int32_t w_dst_dtype);
sf_status sf_pack_weights(const void* w_oihw, int32_t w_src_dtype,
                          int32_t c_out, int32_t c_in, int32_t kernel,
                          int32_t w_dst_dtype, void* w_packed, void* stream);

typedef struct sf_conv_desc {
  int32_t n, c_in, h, w;       /* NCHW input; n folds T*B */
  int32_t c_out, h_out, w_out; /* NCHW output */
  int32_t kernel, stride, padding;  /* (1,1,0), (3,1,1), (3,2,1) */
  int32_t x_dtype;             /* dtype of x and y */
  int32_t w_dtype;             /* dtype of the packed weights: F32 or BF16 */
  int32_t has_bias;            /* bias: fp32 [c_out] */
} sf_conv_desc;

/* Bytes of caller-owned device workspace sf_sparse_conv2d needs (the
 * per-pixel nonzero-channel masks of x: ceil(c_in/64) 64-bit words per pixel,
 * plus one flag word per image). No initialisation is required. */
size_t sf_sparse_conv2d_workspace_size(const sf_conv_desc* d);

/* y = conv2d(x, w) + bias, computed in fp32 over the nonzero input elements
 * only (exact zeros contribute nothing, so skipping them is exact). Two
 * launches: a streaming pass writes the nonzero-channel masks of x into the
 * workspace, then the gather kernel reads masks (and x itself only for
 * images holding values other than 0 and 1). w_packed must be 16-byte
 * aligned; x has no alignment requirement. Patterns: 3x3/s1/p1, 3x3/s2/p1,
 * 1x1/s1/p0 and 1x1/s2/p0 (the last in one pass that builds the masks in
 * shared memory; it uses no workspace). */
sf_status sf_sparse_conv2d(const void* x, const void* w_packed, const float* bias,
                           void* y, const sf_conv_desc* d,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Reads back (synchronously on `stream`) the device error word shared by
 * sf_sparse_conv2d and sf_fused_conv_lif: SF_OK or SF_ERR_DEVICE_TIMEOUT.
 * Not for hot loops. */
sf_status sf_sparse_conv2d_status(void* stream);

/* ------------------------------------------------------------------------ */
/* Fused conv + (BN-folded) bias + LIF over all time steps in one launch.    */
/* ------------------------------------------------------------------------ */
typedef struct sf_lif_desc {
  int32_t t_steps, n, c_in, h, w;   /* x: [t_steps, n, c_in, h, w] */
  int32_t c_out, h_out, w_out;      /* spikes: [t_steps, n, c_out, h_out, w_out] */
  int32_t kernel, stride, padding;
  float tau, v_threshold, v_reset;  /* v_reset is used as 0 when hard_reset == 0 */
  int32_t hard_reset;               /* 1: v = v_reset on spike; 0: v -= v_threshold */
  int32_t decay_input;              /* 1: v += (I - (v - v_reset)) / tau */
  int32_t x_dtype;                  /* dtype of x and of spikes_out */
  int32_t w_dtype;                  /* packed weight dtype: F32 or BF16 */
  int32_t has_bias;
} sf_lif_desc;

/* Workspace bytes of sf_fused_conv_lif (masks of all t_steps * n images). */
size_t sf_fused_conv_lif_workspace_size(const sf_lif_desc* d);

/* v_inout: fp32 [n, c_out, h_out, w_out], read as v[0] and overwritten with
 * the membrane state after the last step. Supports 3x3/s1/p1 and 1x1/s1/p0.
 * spike_masks_out (may be NULL; 8-byte aligned, sf_event_masks_bytes(
 * t_steps * n, c_out, h_out, w_out) bytes): the next layer's events, i.e. the
 * nonzero-channel masks of spikes_out in the layout the mask pass of
 * sf_sparse_conv2d writes ([t_steps*n][h_out][w_out][ceil(c_out/64)] 64-bit
 * words), so the following convolution can run from them
 * (sf_sparse_conv2d_from_masks) without reading the spikes again. */
sf_status sf_fused_conv_lif(const void* x, const void* w_packed, const float* bias,
                            float* v_inout, void* spikes_out, void* spike_masks_out,
                            const sf_lif_desc* d,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of the event masks of n_images images of channels x h x w. */
size_t sf_event_masks_bytes(int64_t n_images, int32_t channels, int32_t h, int32_t w);

/* sf_sparse_conv2d of binary spikes given only their event masks (as written
 * by sf_fused_conv_lif's spike_masks_out; 16-byte aligned): x is not read,
 * no workspace is needed. d->x_dtype is the dtype of y. */
sf_status sf_sparse_conv2d_from_masks(const void* event_masks, const void* w_packed,
                                      const float* bias, void* y, const sf_conv_desc* d,
                                      void* stream);

/* sf_sparse_conv2d of binary spikes x given both x and its event masks: a
 * sampled density of x picks on the device the gather kernel from the masks
 * (sparse spikes) or, for 3x3/s1/p1 layers the tcgen05 kernel takes, the
 * tensor cores reading x; every other shape runs as
 * sf_sparse_conv2d_from_masks. workspace: at least
 * sf_sparse_conv2d_masks_or_x_workspace_size() bytes, 4-byte aligned (the
 * sampled count; ignored where no choice is made). Same reference interface
 * as sf_sparse_conv2d_from_masks. */
size_t sf_sparse_conv2d_masks_or_x_workspace_size(void);
sf_status sf_sparse_conv2d_masks_or_x(const void* x, const void* event_masks, const void* w_packed,
                                      const float* bias, void* y, const sf_conv_desc* d,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Multi-step LIF neuron (the separate LIFNode after a BN, not fused into a  */
/* convolution): the update of Ops/sparse_fused_conv_lif.py:271-293 applied  */
/* over the leading time axis, v kept in registers across all steps.         */
/* ------------------------------------------------------------------------ */
typedef struct sf_lif_ms_desc {
  int64_t numel;                    /* elements per time step (N*C*H*W) */
  int32_t t_steps;
  float tau, v_threshold, v_reset;  /* v_reset is used as 0 when hard_reset == 0 */
  int32_t hard_reset;               /* 1: v = v_reset on spike; 0: v -= v_threshold */
  int32_t decay_input;              /* 1: v += (x - (v - v_reset)) / tau; 0: v += x - (v - v_reset) / tau */
  int32_t x_dtype;                  /* dtype of x */
  int32_t s_dtype;                  /* dtype of spikes_out (values 0 / 1) */
} sf_lif_ms_desc;

/* x: [t_steps, numel]; v_inout: fp32 [numel], read as the state before step 0
 * and overwritten with the state after the last step; spikes_out:
 * [t_steps, numel]. Every pointer device memory, 16-byte alignment enables
 * vector access. No workspace. */
sf_status sf_lif_multistep(const void* x, float* v_inout, void* spikes_out, const sf_lif_ms_desc* d,
                           void* stream);

/* sf_lif_multistep on x viewed as [t_steps][n][c][h][w] (d->numel == n*c*h*w)
 * that also writes the spikes' event masks to spike_masks_out (8-byte aligned,
 * sf_event_masks_bytes(t_steps * n, c, h, w) bytes; every word written): the
 * layout the mask pass of sf_sparse_conv2d writes, so sf_sparse_conv2d_from_masks
 * can run the next convolution without reading the spikes. Spikes and v are
 * identical to sf_lif_multistep's. Reference: the producer-side bitmap of the
 * LIFNode that follows a BN (no fused conv), whose spikes the reference's
 * prescan reads again (Kernels/_prescan_common.py:32-109). */
sf_status sf_lif_multistep_events(const void* x, float* v_inout, void* spikes_out, void* spike_masks_out,
                                  const sf_lif_ms_desc* d, int32_t n, int32_t c, int32_t h, int32_t w,
                                  void* stream);

/* ------------------------------------------------------------------------ */
/* Path policy (process-wide; no counterpart in the reference, whose        */
/* dispatch lives in Kernels/conv2d.py:1026-1178 as fixed Python rules).     */
/* ------------------------------------------------------------------------ */
enum {
  /* 1x1 stride-1 convolutions: 0 automatic (tcgen05 kernel where it applies),
   * 1 two-stage gather path (mask pass + gather kernel), 2 one-pass CUDA-core
   * pointwise kernel. */
  SF_POLICY_CONV1X1_PATH = 0,
  /* Images with fewer pixels than this run 1x1/s1 on the gather kernels
   * (default 128: one MMA tile; smaller maps leave most of a tile empty). */
  SF_POLICY_CONV1X1_TC_MIN_HW = 1,
  /* 3x3 convolutions: 0 automatic, 1 gather kernel only, 2 tcgen05 implicit
   * GEMM wherever it supports the shape. */
  SF_POLICY_CONV3X3_PATH = 2,
  /* 1: sf_lif_multistep_events always uses its general lane-per-pixel kernel. */
  SF_POLICY_LIF_EVENTS_GENERAL = 3,
  /* Fused conv + LIF on the tcgen05 3x3 kernel without event masks: 0
   * automatic (the LIF in the convolution's epilogue, one launch, where the
   * weights stream and one step's images fill the GPU; otherwise the
   * convolution then the multi-step LIF over its output), 1 always the two
   * launches, 2 the epilogue wherever the kernel can stage the membranes. */
  SF_POLICY_LIF_TC_EPILOGUE = 4,
  SF_POLICY_COUNT = 5
};
/* Sets a policy value (>= 0) for every later call in this process. Returns
 * SF_ERR_INVALID_ARG for an unknown key or a negative value. */
sf_status sf_set_path_policy(int32_t key, int64_t value);
/* Current value of a policy key, -1 for an unknown key. */
int64_t sf_get_path_policy(int32_t key);

/* ------------------------------------------------------------------------ */
/* Diagnostics.                                                              */
/* ------------------------------------------------------------------------ */
/* Exercises the bounded-wait path every pipelined kernel here relies on: one
 * thread waits on an mbarrier that nothing arrives on, gives up after
 * limit_ns of wall time and records the timeout. Synchronous on `stream`.
 * Returns SF_ERR_DEVICE_TIMEOUT when the wait expired as it should (and the
 * context is still usable), SF_OK if the barrier completed (a bug), or
 * SF_ERR_CUDA. No counterpart in the reference. */
sf_status sf_selftest_bounded_wait(uint64_t limit_ns, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SPARSEFLOW_B200_H */
