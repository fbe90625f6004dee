/* kirari_b200.h -- C ABI of the B200-native frame path (SPAN x2 upscaler, IFNet interpolator).
 *
 * Drop-in for the reference's upscaler / interpolator engine boundary
 * (Ta2b/Ultimate-Anime-VideoPlayer). The reference boundary is C++-typed -- `gpu::Backend::enqueue
 * (Engine&, span<const Tensor>, span<Tensor>) -> expected<void, Refusal>` (src/gpu/backend.h:438),
 * engines created by `Backend::load` (backend.h:446) and module entry points
 * `kirari_backend_create/destroy` (backend.h:584-587) -- so this header restates it with plain C
 * types: device frame in, device frame out, per-model weights and scales, an int status in place of
 * the named refusal. Nothing here throws, exits or traps; out-of-contract shapes are refused before
 * any launch.
 *
 * Threading: one engine per stream / thread (as the reference's engines, backend.h:445); enqueue is
 * asynchronous on the stream given and never synchronises the host, so it may be captured into a
 * CUDA graph by the caller.
 */
#ifndef KIRARI_B200_H
#define KIRARI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KB2_ABI_VERSION 1

/* Status codes: the reference's RefusalCode values that can cross this boundary
 * (src/core/types.h:21-116), plus KB2_KERNEL_TIMEOUT for a bounded device wait that gave up. */
typedef enum kb2_status {
  KB2_OK = 0,
  KB2_SHAPE_INVALID = 1,        /* RefusalCode::ShapeInvalid: size out of contract */
  KB2_INPUT_MISMATCH = 2,       /* RefusalCode::InputMismatch: wrong tensor count / type / shape */
  KB2_FORMAT_UNSUPPORTED = 3,   /* RefusalCode::FormatUnsupported: model / precision / GPU refused */
  KB2_GPU_MEMORY_EXHAUSTED = 4, /* RefusalCode::GpuMemoryExhausted */
  KB2_VENDOR_CALL_FAILED = 5,   /* RefusalCode::VendorCallFailed: a CUDA call failed */
  KB2_WEIGHTS_INVALID = 6,      /* RefusalCode::HashMismatch / FormatVersion on the weight blob */
  KB2_KERNEL_TIMEOUT = 7,       /* a device-side wait gave up (the kernel returned, context usable) */
  KB2_INVALID_ARGUMENT = 8      /* null pointer or negative count */
} kb2_status;

/* TensorType of src/gpu/tensor.h:10. */
typedef enum kb2_tensor_type { KB2_F32 = 0, KB2_F16 = 1, KB2_U8 = 2, KB2_I8 = 3 } kb2_tensor_type;

/* Tensor of src/gpu/tensor.h:45-50: NCHW shape, device address = handle + offset. */
typedef struct kb2_tensor {
  int32_t type;     /* kb2_tensor_type */
  int64_t dims[4];  /* N, C, H, W */
  uint64_t handle;  /* CUdeviceptr */
  uint64_t offset;  /* bytes */
} kb2_tensor;

/* KB2_MODEL_SPAN_UNSHUFFLE: the AnimeJaNai "unshuffle" SPAN x2 (b5f48, b8f64 ...) of a .span8
 * package (the reference's span_fp8::Package, src/gpu/span_fp8/package.h:1-17, read as
 * span_fp8::parse does, package.cpp:143); `weights` / `weights_bytes` are then the package file's
 * bytes. KB2_PREC_FP16 runs any package in FP16; KB2_PREC_FP8_E4M3 runs an FP8 package's blocks in
 * E4M3 with its own activation scales. Same frames as KB2_MODEL_SPAN_X2 (even H and W). */
/* KB2_MODEL_RIFE_FUSED: RIFE 4.2x (4.25, 4.26, 4.25 lite, 4.22 lite), the reference's fused RIFE
 * (RifeFusedEngine, src/gpu/cuda/backend/rife_fused_engine.h:41; plan src/kernels/spec/rife_fused.h:
 * 7-19) on its native block kernels (src/prepare/rife_native.h). Same enqueue contract as
 * KB2_MODEL_IFNET (image, or the motion variant); weight blob v1 below. */
typedef enum kb2_model {
  KB2_MODEL_SPAN_X2 = 1,
  KB2_MODEL_IFNET = 2,
  KB2_MODEL_SPAN_UNSHUFFLE = 3,
  KB2_MODEL_RIFE_FUSED = 4
} kb2_model;
typedef enum kb2_precision { KB2_PREC_FP16 = 1, KB2_PREC_FP8_E4M3 = 2 } kb2_precision;

typedef struct kb2_engine kb2_engine;

/* Weight blob v1 (KB2_MODEL_SPAN_X2, KB2_MODEL_IFNET and KB2_MODEL_RIFE_FUSED): a 32-byte header,
 * then the network's float32 parameters back to back, little-endian, in the order below. Conv weights are OIHW
 * ([out][in][ky][kx]), transposed-conv weights [in][out][ky][kx] (ONNX ConvTranspose), each
 * followed by its bias and, where the layer has one, its PReLU slopes (one per output channel).
 *
 * KB2_MODEL_SPAN_X2, canonical SPAN x2 (48 channels, 6 blocks; 389,916 floats):
 *   conv_1      W [48][3][3][3],   b [48]
 *   block b = 0..5, conv k = 1..3 (c1, c2 with SiLU after them; c3 into the SPAB gate):
 *               W [48][48][3][3],  b [48]
 *   conv_cat    W [48][192][1][1], b [48]   input channels: [conv_1 out, block 5 out, block 0 out,
 *                                           block 5's c1 activation], 48 each
 *   upsampler   W [12][48][3][3],  b [12]   then PixelShuffle(2), channel c*4 + dy*2 + dx
 *
 * KB2_MODEL_IFNET, classic IFNet (4 blocks at 1/8, 1/4, 1/2, 1/1 with C = 192, 128, 96, 64 channels;
 * 5,160,980 floats). Block k's input has cin = 7 channels for k = 0 (frame A rgb, frame B rgb,
 * timestep) and 12 after (warped A rgb, warped B rgb, timestep, mask, flow 4 / scale), then per block:
 *   conv0a      W [C/2][cin][3][3], b [C/2], slope [C/2]   (stride 2)
 *   conv0b      W [C][C/2][3][3],   b [C],   slope [C]     (stride 2)
 *   res j=0..7  W [C][C][3][3],     b [C],   slope [C]     (PReLU(conv(x) + x))
 *   last        W [C][5][4][4],     b [5]                  (transposed, stride 2, pad 1: 4 flow + mask)
 *
 * KB2_MODEL_RIFE_FUSED, RIFE 4.2x: 12 plan floats first (exact small integers): blocks B (2..5),
 * the input reduction d_0..d_4 of each block (powers of two up to 32, d_0 >= 2, d_(B-1) = 1; 0 past
 * the last block), the block widths C_0..C_4 (32, 64, 96, 128 or 192; 0 past the last block), 16
 * (the encoder width). RIFE 4.25: 5, 8 8 4 2 1, 192 128 96 64 32. Then, with LeakyReLU written
 * as per-channel slopes (0.2 each for the published models):
 *   encoder cnn0 W [16][3][3][3],  b [16], slope [16]   (stride 2)
 *           cnn1 W [16][16][3][3], b [16], slope [16]
 *           cnn2 W [16][16][3][3], b [16], slope [16]
 *           cnn3 W [16][4][4][4],  b [4]                 (transposed, stride 2, pad 1)
 *   block k: cin = 15 for k = 0 (A rgb, B rgb, encodings of A and B, timestep), 28 after (warped A
 *   rgb, warped B rgb, warped encodings of A and B, timestep, mask, 8 attributes, flow 4 / d_k):
 *     conv0a  W [C/2][cin][3][3], b [C/2], slope [C/2]  (stride 2)
 *     conv0b  W [C][C/2][3][3],   b [C],   slope [C]    (stride 2)
 *     res j=0..7 W [C][C][3][3],  b [C],   beta [C], slope [C]   (act(beta (conv(x) + b) + x))
 *     last    W [C][52][4][4],    b [52]                (transposed, stride 2, pad 1; then
 *                                                         DepthToSpace(2, CRD): flow 4, mask, 8)
 */
#define KB2_SPAN_X2_PARAMS 389916
#define KB2_IFNET_PARAMS 5160980

/* The weight blob v1 of KB2_MODEL_RIFE_FUSED from ONNX: the pieces of a split RIFE 4.2x model as the
 * reference's native RIFE path reads them (src/prepare/rife_native.h:39 rife_native_layers, after
 * src/prepare/rife_split.h cut the model): pieces[0] the encoder (cnn0..cnn3), pieces[1 + k] block k,
 * each a ModelProto's bytes whose single input runs through a chain of Conv 3x3 (pad 1, stride 1 or 2)
 * with LeakyRelu / PRelu / Relu, ResConv (Conv, Mul by a per-channel beta, Add of the conv's input,
 * activation) and a last ConvTranspose 4x4 stride 2; Cast and Identity pass through; a 1x1 Conv that
 * follows a conv is folded into it, a depthwise 3x3 stored as a diagonal one (the reference's reader).
 * Initializers and Constant values: FLOAT, FLOAT16, FLOAT8E4M3FN or INT8, raw or typed, inline.
 * reduce[k]: block k's input reduction (the plan: a power of two, 1 to 32; the widths come from the
 * weights), 2 to 5 blocks.
 * blob = NULL: *blob_bytes receives the size; else *blob_bytes is the buffer's capacity on entry and
 * the blob's size on return. Refusals: KB2_WEIGHTS_INVALID (unreadable, or not this topology),
 * KB2_FORMAT_UNSUPPORTED (weights outside the file, segments, sparse initializers, other element
 * types), KB2_INVALID_ARGUMENT; kb2_create_error() says why. Host only: no device is touched. */
int kb2_rife_blob_from_onnx(const void* const* pieces, const uint64_t* piece_bytes, int32_t blocks,
                            const int32_t* reduce, void* blob, uint64_t* blob_bytes);

/* Engine creation parameters (the reference's Artifact + shape set, backend.h:446). */
typedef struct kb2_engine_desc {
  int32_t model;        /* kb2_model */
  int32_t precision;    /* kb2_precision (IFNet: FP16 only) */
  int32_t max_batch;    /* frames (SPAN) or frame pairs (IFNet) per enqueue, >= 1 */
  int32_t height;       /* input frame height */
  int32_t width;        /* input frame width */
  int32_t device;       /* CUDA device ordinal */
  const void* weights;  /* weight blob v1, host memory: 32-byte header ("KB2WGT01", u32 version 1,
                           u32 model, u64 float count, u32 CRC-32 of the payload, u32 0), then the
                           float32 parameters in the model's order */
  uint64_t weights_bytes;
  const float* act_scales; /* FP8: per-tensor E4M3 activation scales (SPAN: 19), host memory */
  int32_t act_scale_count;
} kb2_engine_desc;

/* Module identity (replaces kirari_backend_abi, src/gpu/backend.h:584). */
int kb2_abi_version(void);

/* Creates an engine: validates the blob (magic, version, CRC-32, parameter count), packs the weights
 * for the tensor cores, allocates the activation workspace. Replaces Backend::load
 * (src/gpu/backend.h:446) for SpanFp8Engine (src/gpu/cuda/backend/span_fp8_engine.h:45) and
 * RifeFusedEngine (rife_fused_engine.h:41). On failure *out is null and the status says why;
 * kb2_create_error() returns the message. */
int kb2_create(const kb2_engine_desc* desc, kb2_engine** out);
const char* kb2_create_error(void);

/* Destroys an engine (waits for its device work). Replaces the Engine destructor. */
int kb2_destroy(kb2_engine* engine);

/* Last refusal message of this engine ("" if none). */
const char* kb2_last_error(const kb2_engine* engine);

/* Device bytes the engine owns (weights + workspace), as SpanFp8Net::workspace_bytes
 * (src/gpu/cuda/backend/span_fp8_net.h:136). */
int kb2_workspace_bytes(const kb2_engine* engine, uint64_t* bytes);

/* Enqueues one pass on `stream` (a cudaStream_t; 0 = legacy default stream). Replaces
 * Backend::enqueue (src/gpu/backend.h:438) -> TensorRtBackend::enqueue_span_fp8 / enqueue_rife_fused
 * (src/gpu/cuda/backend/tensorrt_backend.cpp:527-548).
 *   SPAN:  inputs[0] = F16 [n,3,H,W];              outputs[0] = F16 [n,3,2H,2W]
 *   IFNet: inputs[0] = F16 [n,3,H,W] (frame A), inputs[1] = F16 [n,3,H,W] (frame B);
 *          outputs[0] = F16 [n,3,H,W] (the frame at the engine's timestep), or, the motion
 *          variant (the reference's run_motion, src/app/play/upscale_motion.cpp:71-84, whose finish
 *          writes "flow and mask", src/gpu/cuda/backend/rife_finish.cuh:40-55): two outputs
 *          outputs[0] = flow [n,4,Hp,Wp] (f0x, f0y, f1x, f1y: displacements to frames A and B in
 *          pixels) and outputs[1] = mask [n,1,Hp,Wp] (sigmoid of the mask: the weight of frame A),
 *          both F32 or both F16, over the padded plane of kb2_rife_geometry. F32 outputs feed
 *          kb2_motion (kb2_warp_blend_at, kb2_flow_max) directly.
 * n <= max_batch, H and W the engine's. Device pointers must be 16-byte aligned. */
int kb2_enqueue(kb2_engine* engine, void* stream, const kb2_tensor* inputs, int32_t n_inputs,
                const kb2_tensor* outputs, int32_t n_outputs);

/* SPAN x2: what the following enqueues write. 0 (the default): F16 frames [n,3,2H,2W]. A
 * kb2_display_format: the display pixels the reference's ring store writes from its last layer's
 * epilogue (store_pixel, src/gpu/cuda/backend/span_native16_kernels.cuh:325; pixel codes of
 * src/kernels/spec/ring_pack.h), written here by the upsampler's epilogue, with no F16 frame in
 * between: outputs[0] is then U8 [n, B, 2H, 2W] with B = 8 (RGBA16) or 4 (RGB10A2 forms) bytes a
 * pixel, the pixels packed row by row (row pitch 2W * B bytes; the C dimension is the pixel's bytes,
 * interleaved). Each pixel equals kb2_pack_display of the F16 frame the engine would have written.
 * KB2_FORMAT_UNSUPPORTED for other engines. */
int kb2_set_output_format(kb2_engine* engine, int32_t format);

/* SPAN x2: process every frame of the following enqueues as `tiles` row tiles (configs[2] of the
 * contract: 8 tiles with an 8-pixel halo), the way a player that runs SPAN on bands of rows does.
 * Tile t owns the core rows [t * C, min(H, (t + 1) * C)), C = ceil(H / tiles), and is computed from
 * C + 2 * halo input rows around them (the window moved inside the frame at its top and bottom),
 * as one frame of zero-padded SPAN; the tiles' core output rows are stitched into outputs[0]. The
 * network's receptive radius is 20 input rows (conv_1, three 3x3 convs a block, the upsampler), so
 * a halo of 20 or more gives the whole-frame result (up to the order of FP32 sums), a smaller one
 * changes the rows near the seams (the reference's exact_side, src/gpu/span_fp8/forward.cpp:169,
 * states the same bound). tiles <= 1: whole frames (the default). Builds a second network of the
 * tile's height (device memory); 1 <= tiles <= H / 2, 0 <= halo <= 64, else KB2_SHAPE_INVALID. */
int kb2_set_row_tiles(kb2_engine* engine, int32_t tiles, int32_t halo);

/* Moving tiles of SPAN x2 (the reference's kernels/spec/span_tiles.h, Engine::span_tile_grid and
 * Engine::next_span_tiles, src/gpu/backend.h:401-412): only the tiles that changed are recomputed,
 * the rest of the output keeps the previous frame's. The grid is in input pixels: tile_w x tile_h
 * tiles from (0, 0), row by row, the last row and column cut by the frame; reach_* is the network's
 * receptive radius (20 input pixels) rounded up to tiles: the caller marks as core every tile whose
 * output can change, i.e. within reach of a changed input pixel (kernels::dilate_span_tiles). */
typedef struct kb2_tile_grid {
  int32_t tile_w, tile_h; /* input pixels */
  int32_t cols, rows;     /* tiles across and down */
  int32_t reach_cols, reach_rows;
  int32_t shift_step;     /* a pan must be a multiple of this many input pixels */
  int32_t scale;          /* output pixels per input pixel (2) */
} kb2_tile_grid;
int kb2_span_tile_grid(const kb2_engine* engine, kb2_tile_grid* grid);

/* The next kb2_enqueue of this SPAN x2 engine (one call only) computes only what the tiles marked
 * non-zero in `core` (cols x rows bytes, row by row) need, and writes outputs[0] only there. Before
 * that, if `previous` is not null and is not the call's output, outputs[0] receives `previous` (the
 * previous call's output, same type and shape) moved by (shift_x, shift_y) input pixels (x scale
 * output pixels), its pixels whose source falls outside the frame left as they are (their tiles must
 * be core); `previous` null: outputs[0] already holds the previous output, and there is no shift. A
 * shift onto the same buffer makes the next call compute and write the whole frame. The engine
 * computes each dirty row of tiles from a window of its rows plus the reach above and below, or the
 * whole frame when that costs less; the core tiles' values equal the whole frame's up to the order of
 * FP32 sums. KB2_OK: the next call will do it; KB2_FORMAT_UNSUPPORTED (an empty core, which cancels a
 * pending request; a shift without `previous`; row tiles on; another model): the next call computes
 * the whole frame. The first request allocates the window network (device memory). */
int kb2_next_span_tiles(kb2_engine* engine, const uint8_t* core, int32_t count, int32_t shift_x, int32_t shift_y,
                        const kb2_tensor* previous);

/* IFNet: the padded plane the network runs on (multiples of 32) and the frame's window in it, as the
 * reference's rife_geometry (src/kernels/spec/rife.h:47-63; left / top = half the padding, rounded
 * down to even): the motion outputs are plane_h x plane_w, the frame at (window_x, window_y). */
int kb2_rife_geometry(const kb2_engine* engine, int32_t* plane_h, int32_t* plane_w, int32_t* window_x,
                      int32_t* window_y);

/* IFNet: timestep of the following enqueues, in (0, 1) (the time planes of the reference's
 * 11-plane input, src/kernels/spec/rife.h:60; Engine::next_times_only, backend.h:391). */
int kb2_set_timestep(kb2_engine* engine, float timestep);

/* Reads and clears the engine's device error word after synchronising `stream`: KB2_OK, or
 * KB2_KERNEL_TIMEOUT with the code in *code (which wait gave up). */
int kb2_check_device(kb2_engine* engine, void* stream, int32_t* code);

/* No counterpart in the reference. Self-test of the bounded device waits behind KB2_KERNEL_TIMEOUT:
 * on `device`, one thread waits on a barrier that nothing completes, through the same wait every
 * kernel of this library uses; the wait gives up after its time limit (2 s), records its code and
 * the kernel ends normally. Returns KB2_KERNEL_TIMEOUT with the code (0x500) in *code and the time
 * the device waited in *waited_seconds (either may be null); the device stays usable. Blocks the
 * calling thread for that time; allocates 16 bytes of device memory. */
int kb2_selftest_bounded_wait(int32_t device, int32_t* code, double* waited_seconds);

/* SPAN FP16 engines only: runs the frames through the FP16 network and returns, per quantised tensor,
 * the maximum |value| seen, the calibration of span_fp8::derive (src/gpu/span_fp8/derive.h:42-46).
 * KB2_MODEL_SPAN_X2: 19 peaks ([3b] block b input, [3b+1] / [3b+2] its two activations, [18] last
 * block output). KB2_MODEL_SPAN_UNSHUFFLE: 1 + 3 * blocks peaks in the package's scale order
 * (package.h:15-17: conv_1's output, then per block its two ReLU outputs and its output), so that a
 * player derives an FP8 package from an FP16 one on the device. Synchronous on `stream`. Scales are
 * then peak * 1.25 / 448. */
int kb2_span_calibrate(kb2_engine* engine, void* stream, const kb2_tensor* frames, float* peaks,
                       int32_t n_peaks);

/* kb2_span_calibrate without any device allocation. This entry point has no counterpart in the
 * reference: it exists for callers that reserve all their device memory up front and cannot let a
 * call allocate. kb2_span_calibrate allocates scratch for the discarded x2 output frames on every
 * call; this variant takes it, and the 19 peak words, from a 64 MiB __device__ array compiled into
 * the library (one per device, shared by all engines on it).
 *   - Same arguments, checks and result as kb2_span_calibrate. Peaks are bit-identical.
 *   - Limit: one x2 output frame (24 * H * W bytes) plus 256 bytes must fit in 64 MiB, i.e.
 *     H * W <= 2,796,192 pixels (1920x1080 fits, 2560x1440 does not); larger engines are refused
 *     with KB2_SHAPE_INVALID. Frames run min(max_batch, what fits) at a time.
 *   - The engine's device must be the current device. Every call looks up the array's address in
 *     the current context (cudaGetSymbolAddress); the first call in a context makes the driver load
 *     and reserve it there: make that first call before any stream capture begins. Under lazy
 *     module loading (CUDA's default) only that first call reserves the 64 MiB; with
 *     CUDA_MODULE_LOADING=EAGER every context that loads this library reserves it on each device it
 *     uses, whether or not this entry point is called. The call is synchronous on `stream`.
 *   - Profiling must be off (its timing events would be created on demand).
 *   - Overlapping calls on one device race on the shared array: serialise them. */
int kb2_span_calibrate_static(kb2_engine* engine, void* stream, const kb2_tensor* frames, float* peaks,
                              int32_t n_peaks);

/* The warp tap rule of the IFNet path, on the device, for callers and tests that need the exact
 * sample positions: for a flow field [n][2][h][w] (FP32, device memory; plane 0 = x, plane 1 = y)
 * writes x0, x1, y0, y1 as int32 planes [n][4][h][w] and the weights wx, wy as FP32 planes
 * [n][2][h][w] of the bilinear backward warp over the whole h x w plane. The rule is the reference's
 * tap_at (src/gpu/cuda/backend/warp_lib.cuh:45-58, src/kernels/spec/warp.h:44-49): ix = x + fx in
 * FP32 round-to-nearest, clamped to [0, w - 1] (NaN to 0), x0 = trunc(ix), x1 = min(x0 + 1, w - 1),
 * wx = ix - x0; the same along y. Asynchronous on `stream`. */
int kb2_warp_taps(void* stream, const float* flow, int32_t n, int32_t h, int32_t w, int32_t* taps, float* weights);

/* Per-layer device timing, the role of the reference's GpuTiming event pairs
 * (src/gpu/cuda/backend/gpu_timing.h:1-40): while enabled, every kernel launch of an enqueue is
 * bracketed by CUDA events on the enqueue's stream; kb2_read_profile synchronises the engine's last
 * stream and returns one record per layer kind, accumulated since profiling was enabled. */
typedef struct kb2_layer_profile {
  char name[48];         /* layer kind, e.g. "span.block_conv.fp16.silu" */
  uint64_t launches;     /* launches timed */
  double total_ms;       /* summed device time */
  double flops;          /* algorithmic FLOPs per launch (direct-conv MACs x 2), averaged over the launches */
  double bytes;          /* algorithmic HBM bytes per launch (inputs + outputs once), averaged likewise */
} kb2_layer_profile;

/* Motion of frame pairs at their middle, as RIFE estimates it (the reference's kernels::ref::Motion,
 * src/kernels/ref/warp.h:16-28): `flow` device FP32 [n][4][plane_h][plane_w] (f0x, f0y, f1x, f1y:
 * displacements to frame a and to frame b, in pixels of the window), `mask` device FP32
 * [n][plane_h][plane_w] (weight of frame a), and the frames' window in those planes. */
typedef struct kb2_motion {
  const float* flow;
  const float* mask;
  int32_t plane_h, plane_w;
  int32_t x, y, width, height;
  int32_t warp;     /* the filter that reads frames a and b: 0 bilinear, 1 Catmull-Rom (RifeWarp) */
  int32_t pan_lock; /* 1: estimate each pair's global translation on a and b and use it where RIFE's flow
                       is small and close to it, fading to a linear blend under half a pixel of motion
                       (Motion::pan_lock, spec/warp_pan.h); at most 64 pairs a call, whose estimates
                       share a static device array: pan-locked calls that overlap on the GPU race; not
                       with keep-poses */
  int32_t at_instant; /* 1: the motion was estimated at the output instant (RIFE run at t directly):
                         read as it is at any t, without the straight-line step or the blend law */
} kb2_motion;

/* Frames at instant t in (0, 1) from frames a, b (F16 [n,3,H,W], device) and their mid-pair
 * motion, into out (F16 [n,3,H,W]); asynchronous on `stream`. Replaces warp_blend_at
 * (src/kernels/ref/warp.cpp:261; its CUDA form k_warp_blend_mid): t = 1/2 reads flow and mask as
 * they are; other t move each point on a straight line from the middle and weight a by the blend law
 * logit(m) = logit(mask) + 2.591 ln((1 - t) / t) (src/kernels/spec/warp.h:58-74). Bilinear reads. */
int kb2_warp_blend_at(void* stream, const kb2_tensor* a, const kb2_tensor* b, const kb2_motion* motion, float t,
                      const kb2_tensor* out);

/* kb2_warp_blend_at that keeps the poses (warp_blend_poses, src/kernels/ref/warp.cpp:270;
 * src/kernels/spec/poses.h): each pixel's instant is adjusted by the ratio of the distance its point
 * moved in the previous pair (`previous`, the same planes and window; null for a held pair) to the
 * one it moves now, so that a character animated on twos keeps its pose over a panning background. */
int kb2_warp_blend_poses(void* stream, const kb2_tensor* a, const kb2_tensor* b, const kb2_motion* motion,
                         const kb2_motion* previous, float t, const kb2_tensor* out);

/* Per frame pair, the 99.9th percentile of the largest |flow component| over the window, in pixels of
 * the window (flow_max, src/kernels/ref/warp.cpp:290: the test for one RIFE pass per calm pair,
 * src/kernels/spec/warp.h:76-110). bins: the caller's device scratch of n x 256 uint32; out: host
 * float[n]. Synchronises `stream`. */
int kb2_flow_max(void* stream, const kb2_motion* motion, int32_t n, uint32_t* bins, float* out);

/* Display-ring pixel formats (the reference's RingPacking; src/kernels/spec/ring_pack.h). */
typedef enum kb2_display_format {
  KB2_DISPLAY_RGBA16 = 1,        /* 4 x u16 UNORM, alpha 65535 (8 bytes a pixel) */
  KB2_DISPLAY_RGB10A2 = 2,       /* r | g << 10 | b << 20 | 3 << 30, 10-bit UNORM (4 bytes a pixel) */
  KB2_DISPLAY_RGB10A2_DITHER = 3 /* the same with the pixel's fixed TPDF dither before truncation */
} kb2_display_format;

/* Packs frames (F16 [n,3,H,W], device, e.g. an engine's output) into display pixels: frame f row y
 * at out + (f * H + y) * pitch bytes (device). The reference's ring store (store_ring,
 * src/gpu/cuda/backend/pixel_kernels.cuh:78; contract src/kernels/spec/ring_pack.h and color.h
 * unorm16): clamp to [0, 1] (NaN to 0), x 65535 or x 1023, + 0.5, truncate. Asynchronous on stream. */
int kb2_pack_display(void* stream, const kb2_tensor* frames, int32_t format, void* out, int64_t pitch);

int kb2_set_profiling(kb2_engine* engine, int32_t enable);
int kb2_read_profile(kb2_engine* engine, kb2_layer_profile* records, int32_t capacity, int32_t* count);
/* Kernel launches one enqueue issues (all of them this library's own kernels). */
int kb2_launches_per_enqueue(const kb2_engine* engine, int32_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* KIRARI_B200_H */
