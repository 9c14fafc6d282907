/*
 * fussim_b200 — C ABI of the B200 SSIM loss engine.
 *
 * Plain pointers and sizes only; no C++ or torch types cross this boundary. Every
 * entry point is asynchronous on the given stream, never throws, and returns a
 * fssim_status (0 = success). Tensors are dense NCHW (B, C, H, W) in device memory,
 * element offsets computed in 64-bit.
 *
 * Two families of entry points:
 *
 *  1. The five reference extension functions of OpsiClear/fussim, one C function each,
 *     with the same argument meaning and outputs (csrc/ext.cpp:11-17). A binding that
 *     today calls the reference's pybind module can call these instead.
 *
 *  2. The fused loss path used by fussim_b200.fused_ssim / ssim / SSIM: a forward that
 *     writes the three SSIM partials and a deterministic in-kernel mean (or per-image
 *     means) without materialising the SSIM map, and a backward that applies the
 *     transposed Gaussian with the upstream gradient folded in as a per-image scalar.
 *
 * Window sizes 7, 9 and 11 use the reference's Gaussian tables (csrc/ssim.cu:28-64);
 * the FP16-input entry points use those tables rounded to half precision
 * (csrc/ssim_fp16.cu:55-82). All arithmetic is FP32.
 */
#ifndef FUSSIM_B200_H_
#define FUSSIM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same layout as cudaStream_t; pass NULL for the legacy default stream. */
typedef struct CUstream_st* fssim_stream_t;

typedef enum fssim_status {
  FSSIM_OK = 0,
  FSSIM_ERR_WINDOW = 1,      /* window_size not in {7, 9, 11} */
  FSSIM_ERR_SHAPE = 2,       /* a dimension is negative or too large */
  FSSIM_ERR_DTYPE = 3,       /* unsupported element-type combination */
  FSSIM_ERR_NULLPTR = 4,     /* a required pointer is NULL */
  FSSIM_ERR_WORKSPACE = 5,   /* workspace missing or too small */
  FSSIM_ERR_CUDA = 6,        /* a CUDA runtime call or kernel launch failed */
  FSSIM_ERR_ARGUMENT = 7     /* any other invalid argument */
} fssim_status;

typedef enum fssim_dtype {
  FSSIM_F32 = 0,
  FSSIM_F16 = 1,
  FSSIM_BF16 = 2
} fssim_dtype;

/* Human-readable text for a status code. */
const char* fssim_status_string(int status);

/* Detail of the last error raised on the calling thread ("" if none). */
const char* fssim_last_error(void);

/* Library version, e.g. "0.1.0". */
const char* fssim_version(void);

/* Failures detected inside the kernels on the current device since the flag was last
 * cleared, as a bit set (0 = none). Synchronises with the device. clear != 0 resets the flag.
 *  Bit 0: a kernel's input staging did not complete within its bounded wait. The CTA that
 *         gave up stops; a forward with a reduction still completes its reduction, writes
 *         NaN to every reduced output of that call (out, image_sums, a sharded rank's
 *         published sum) and leaves its workspace zero-filled, so the next call on the same
 *         workspace is unaffected. Per-pixel outputs (map, partials, gradient) of the
 *         failed call are incomplete.
 *  Bit 1: fssim_dp_gather gave up waiting for another rank (see section 3); it wrote NaN. */
int fssim_poll_device_error(unsigned* code, int clear);

/* Polls of a staging step's wait before the step gives up (bit 0 above). polls < 0 restores
 * the default (2^20 polls, milliseconds). polls == 0 makes every step that is staged by the
 * tensor memory accelerator give up at once: a way to exercise the failure path. Applies to
 * launches made after the call; process-wide. */
int fssim_set_staging_wait_limit(long long polls);

/* How long fssim_dp_gather waits for the other ranks before it gives up (bit 1 above), in
 * microseconds of the device's global timer. us <= 0 restores the default (10 s).
 * Applies to launches made after the call; process-wide. */
int fssim_set_gather_timeout_us(long long us);

/* Kernels of the fused loss path (fssim_forward, fssim_backward and the sharded forward).
 * Both families compute bitwise-identical per-pixel results (partials, gradients, maps):
 *  FSSIM_KERNELS_STREAM: 64-thread CTAs, one output column per thread, the vertical filter
 *      window carried in registers from step to step;
 *  FSSIM_KERNELS_TILE: 128-thread CTAs computing 2-column x 4-row tiles, the vertical halo
 *      kept in shared memory (the kernels of the map entry points in section 1);
 *  FSSIM_KERNELS_AUTO (default): per launch, the family measured faster on a B200 for its
 *      size: the streaming kernels, except the tile kernels below 2^21 channel-pixels
 *      (B*C*H*W) and the tile backward from 2^27 channel-pixels.
 * Process-wide; applies to launches made after the call (FSSIM_ERR_ARGUMENT otherwise). */
#define FSSIM_KERNELS_STREAM 0
#define FSSIM_KERNELS_TILE 1
#define FSSIM_KERNELS_AUTO 2
int fssim_set_loss_kernels(int family);

/* Number of SMs the kernels' persistent grids leave unused (default 0), for callers that
 * run another kernel concurrently, e.g. a collective overlapping the backward: a grid that
 * fills every SM would otherwise wait for that kernel's blocks to leave before its last
 * CTAs start. Process-wide; n >= 0 (FSSIM_ERR_ARGUMENT otherwise). */
int fssim_set_reserved_sms(int n);

/* ------------------------------------------------------------------------------------
 * 1. Reference extension functions (map-producing compat seam)
 * ------------------------------------------------------------------------------------ */

/* Replaces fusedssim() (csrc/ssim.h:12-20, dispatch csrc/ssim.cu:603-619).
 * img1/img2: FP32 (B,C,H,W). Writes ssim_map (FP32, B*C*H*W) and, when train != 0, the
 * three partials dm_dmu1, dm_dsigma1_sq, dm_dsigma12 (FP32, B*C*H*W each; may be NULL
 * when train == 0). */
int fssim_fusedssim(int window_size, float C1, float C2, const float* img1, const float* img2,
                    int64_t B, int64_t C, int64_t H, int64_t W, int train, float* ssim_map,
                    float* dm_dmu1, float* dm_dsigma1_sq, float* dm_dsigma12,
                    fssim_stream_t stream);

/* Replaces fusedssim_backward() (csrc/ssim.h:22-33, dispatch csrc/ssim.cu:621-640).
 * dL_dimg1(p) = sum_q w(q-p) * dL_dmap(q) * [dm_dmu1 + 2 img1(p) dm_dsigma1_sq
 *                                           + img2(p) dm_dsigma12](q). All FP32. */
int fssim_fusedssim_backward(int window_size, float C1, float C2, const float* img1,
                             const float* img2, const float* dL_dmap, const float* dm_dmu1,
                             const float* dm_dsigma1_sq, const float* dm_dsigma12, int64_t B,
                             int64_t C, int64_t H, int64_t W, float* dL_dimg1,
                             fssim_stream_t stream);

/* Replaces fusedssim_fp16() (csrc/ssim_fp16.h:14-20, csrc/ssim_fp16.cu:791-805).
 * img1/img2: IEEE half bit patterns. Writes the FP32 ssim_map. */
int fssim_fusedssim_fp16(int window_size, float C1, float C2, const uint16_t* img1,
                         const uint16_t* img2, int64_t B, int64_t C, int64_t H, int64_t W,
                         float* ssim_map, fssim_stream_t stream);

/* Replaces fusedssim_fp16_train() (csrc/ssim_fp16.h:22-31, csrc/ssim_fp16.cu:807-822).
 * Half inputs; FP32 map and FP32 partials. */
int fssim_fusedssim_fp16_train(int window_size, float C1, float C2, const uint16_t* img1,
                               const uint16_t* img2, int64_t B, int64_t C, int64_t H,
                               int64_t W, float* ssim_map, float* dm_dmu1,
                               float* dm_dsigma1_sq, float* dm_dsigma12,
                               fssim_stream_t stream);

/* Replaces fusedssim_fp16_backward() (csrc/ssim_fp16.h:33-44, csrc/ssim_fp16.cu:824-842).
 * Half images; FP32 dL_dmap and partials; FP32 gradient. */
int fssim_fusedssim_fp16_backward(int window_size, float C1, float C2, const uint16_t* img1,
                                  const uint16_t* img2, const float* dL_dmap,
                                  const float* dm_dmu1, const float* dm_dsigma1_sq,
                                  const float* dm_dsigma12, int64_t B, int64_t C, int64_t H,
                                  int64_t W, float* dL_dimg1, fssim_stream_t stream);

/* ------------------------------------------------------------------------------------
 * 2. Fused loss path
 * ------------------------------------------------------------------------------------ */

typedef enum fssim_reduce {
  FSSIM_REDUCE_NONE = 0,      /* no reduction outputs */
  FSSIM_REDUCE_SCALAR = 1,    /* out[0] = out_scale * sum over the whole batch */
  FSSIM_REDUCE_PER_IMAGE = 2  /* out[b] = out_scale * sum over image b */
} fssim_reduce;

typedef struct fssim_forward_args {
  int32_t dtype;          /* fssim_dtype of img1 and img2 (F32 or F16) */
  int32_t partial_dtype;  /* fssim_dtype of the partials (F32, or F16 with F16 images) */
  int64_t B, C, H, W;
  int32_t window_size;    /* 7, 9 or 11 */
  int32_t valid;          /* 0: 'same' zero padding; 1: 'valid' (border of (w-1)/2 cropped) */
  int32_t clamp;          /* 1: clamp the map at 0 before reducing (nonnegative_ssim) */
  int32_t train;          /* 1: write the partials */
  int32_t reduce;         /* fssim_reduce */
  float C1, C2;
  float out_scale;        /* multiplies the reduced sums (e.g. 1/count) */
  const void* img1;
  const void* img2;
  /* Optional per-pixel outputs (NULL to skip): */
  float* ssim_map;        /* B*C*H*W FP32: the uncropped, unclamped map */
  void* partials;         /* 3*B*C*H*W of partial_dtype: dm_dmu1 | dm_dsigma1_sq | dm_dsigma12.
                           * Pre-masked for the fused backward: zero outside the valid
                           * crop and where the clamp is active. */
  /* Reduction outputs (required when reduce != NONE): */
  float* out;             /* 1 (SCALAR) or B (PER_IMAGE) FP32 values */
  double* image_sums;     /* optional: B FP64 per-image sums of the (cropped, clamped) map */
  /* Scratch for the reduction: fssim_forward_workspace_bytes(B) bytes, zero-filled before
   * its first use. Every call leaves it zero-filled again, so it can be reused by later
   * calls on the same stream; calls that may overlap on the GPU need separate workspaces. */
  void* workspace;
  size_t workspace_bytes;
  /* Fused L1 term (the 3DGS loss (1-l)*mean|x-y| + l*(1-SSIM)): with l1_weight != 0 (and a
   * reduction) the forward also sums |img1 - img2| over every pixel of each image and
   * writes out = out_scale * sum(ssim) + l1_weight * sum|img1 - img2| + out_offset (per
   * image for FSSIM_REDUCE_PER_IMAGE). Zero-initialise both for plain SSIM. */
  float l1_weight;
  float out_offset;
} fssim_forward_args;

typedef struct fssim_backward_args {
  int32_t dtype;          /* fssim_dtype of img1/img2 */
  int32_t partial_dtype;  /* fssim_dtype of the partials */
  int32_t grad_dtype;     /* fssim_dtype of the gradient written to grad */
  int64_t B, C, H, W;
  int32_t window_size;
  const void* img1;
  const void* img2;
  const void* partials;   /* as written by fssim_forward (3*B*C*H*W) */
  /* dL/dmap(pixel of image b) = chain_scale * grad_out[per_image ? b : 0]
   * (grad_out == NULL reads as 1). grad_out is an FP32 device pointer. */
  const float* grad_out;
  int32_t grad_out_per_image;
  float chain_scale;
  void* grad;             /* B*C*H*W of grad_dtype */
  /* Fused L1 term: adds l1_scale * grad_out[.] * sign(img1 - img2) (0 where equal) to every
   * pixel's gradient. 0 for plain SSIM. */
  float l1_scale;
} fssim_backward_args;

/* Bytes of workspace fssim_forward needs for a batch of B images. */
size_t fssim_forward_workspace_bytes(int64_t B);

/* Fused forward. New in this engine; it replaces the reference's sequence
 * fusedssim() + valid crop + ssim_map.mean() (fussim/__init__.py:363-369,580). */
int fssim_forward(const fssim_forward_args* args, fssim_stream_t stream);

/* Fused backward. Replaces the reference's sequence expand(dL/dmean) + valid zero
 * scatter + fusedssim_backward() (fussim/__init__.py:381-395). */
int fssim_backward(const fssim_backward_args* args, fssim_stream_t stream);

/* Largest batch fssim_forward_noalloc accepts. */
#define FSSIM_NOALLOC_MAX_IMAGES 4096

/* fssim_forward for callers that cannot allocate GPU memory (no counterpart in the
 * reference). Same arguments and outputs as fssim_forward; args->workspace and
 * args->workspace_bytes are ignored. The reduction scratch is a fixed array in the
 * library's device memory (about 65 KiB, held by every GPU that loads the library until
 * exit), so nothing is allocated per call: for plugins whose host owns all device memory,
 * fixed-budget real-time loops, and bindings without a device allocator. Limits: at most
 * FSSIM_NOALLOC_MAX_IMAGES images (larger B returns FSSIM_ERR_WORKSPACE); all calls share
 * the array, so calls that overlap on the GPU race and must be serialised; the first call
 * on each device performs a one-time set-up (cudaGetSymbolAddress) and should come before
 * any stream capture on that device. */
int fssim_forward_noalloc(const fssim_forward_args* args, fssim_stream_t stream);

/* ------------------------------------------------------------------------------------
 * 3. Batch-sharded loss over several GPUs (one process per GPU, no counterpart in the
 *    reference). The global mean over all ranks' shards is formed without a collective
 *    library call: the forward's last CTA stores the rank's sum into every rank's mailbox
 *    over NVLink (CUDA IPC mappings), and a one-warp gather kernel on each rank sums the
 *    world values in rank order (identical bits on every rank).
 *
 *    Set-up, once per group: each rank allocates its mailbox (fssim_dp_mailbox_alloc),
 *    exports it (fssim_ipc_get_handle), exchanges the handles with the other ranks by any
 *    host channel, and maps the peers' mailboxes (fssim_ipc_open_handle).
 *    Per step: every rank calls fssim_forward_dp with the same seq (1, 2, 3, ...), then
 *    fssim_dp_gather. The gather waits for the other ranks for at most the time set by
 *    fssim_set_gather_timeout_us (default 10 s); on time-out it writes NaN and sets bit 1
 *    of fssim_poll_device_error. A rank that falls further behind (e.g. while it writes a
 *    checkpoint) must first bring the others to a host-side barrier.
 * ------------------------------------------------------------------------------------ */

#define FSSIM_DP_MAX_RANKS 8
#define FSSIM_IPC_HANDLE_BYTES 64

typedef struct fssim_dp_args {
  int32_t world;                          /* ranks (1..FSSIM_DP_MAX_RANKS) */
  int32_t rank;                           /* this rank */
  uint64_t seq;                           /* step number, >= 1, the same on every rank */
  void* mailboxes[FSSIM_DP_MAX_RANKS];    /* mailbox of rank r as mapped in this process */
} fssim_dp_args;

/* Bytes of one mailbox for `world` ranks. */
size_t fssim_dp_mailbox_bytes(int world);

/* Allocates (cudaMalloc, a whole allocation) and zero-fills this rank's mailbox on the
 * current device; fssim_dp_mailbox_free releases it. */
int fssim_dp_mailbox_alloc(int world, void** mailbox);
int fssim_dp_mailbox_free(void* mailbox);

/* CUDA IPC export of a mailbox, and mapping / unmapping of a peer's exported mailbox. */
int fssim_ipc_get_handle(const void* mailbox, unsigned char handle[FSSIM_IPC_HANDLE_BYTES]);
int fssim_ipc_open_handle(const unsigned char handle[FSSIM_IPC_HANDLE_BYTES],
                          void** peer_mailbox);
int fssim_ipc_close_handle(void* peer_mailbox);

/* fssim_forward of this rank's shard (reduce must be FSSIM_REDUCE_SCALAR), which also
 * publishes the shard's FP64 sum to every rank's mailbox. out[0] receives the local
 * out_scale * sum; fssim_dp_gather replaces it with the global value. */
int fssim_forward_dp(const fssim_forward_args* args, const fssim_dp_args* dp,
                     fssim_stream_t stream);

/* out[0] = scale * (sum of the world ranks' published sums of step dp->seq, rank order). */
int fssim_dp_gather(const fssim_dp_args* dp, float scale, float* out, fssim_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FUSSIM_B200_H_ */
