/*
 * illumina.h -- C ABI of the B200-native IlluminaDepth hot path.
 *
 * One shared library (libillumina.so) replaces the reference's WebGPU runner,
 * kernels and lighting pass. Every entry point is plain C: pointers, sizes and
 * status codes, no C++ or torch types. A node-api addon (or any FFI) binds
 * them 1:1 and turns a non-OK status into `throw new Error(illumina_last_error())`.
 *
 * Pointers: frame, disparity and tensor arguments may be host memory (pageable
 * or pinned) or device memory of the model's device, unless an entry point says
 * "device". `stream` is a cudaStream_t (NULL = the legacy default stream).
 *
 * Threading: one model per device; calls on one model are not re-entrant. Use
 * one host thread per device for multi-GPU work. illumina_last_error() is
 * thread-local.
 *
 * Each declaration names the reference interface it replaces (file:line within
 * the reference project).
 */
#ifndef ILLUMINA_H
#define ILLUMINA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The message for the last failure on this thread is in
 * illumina_last_error(); weight errors use the reference's wording
 * (src/model/weights.ts:97-165). */
typedef enum illumina_status {
  ILLUMINA_OK = 0,
  ILLUMINA_INVALID_ARG = 1,
  ILLUMINA_BAD_WEIGHTS = 2,
  ILLUMINA_ARCH_MISMATCH = 3,
  ILLUMINA_CUDA_ERROR = 4,
  ILLUMINA_TIMEOUT = 5,
  ILLUMINA_NO_DEVICE = 6
} illumina_status;

/* Activation ids (src/model/arch.ts:32, src/model/layout.ts:131-142). */
enum { ILLUMINA_ACT_LINEAR = 0, ILLUMINA_ACT_RELU = 1, ILLUMINA_ACT_RELU6 = 2, ILLUMINA_ACT_HARDSWISH = 3 };

/* Arithmetic of the network: fp32 everywhere, or bf16 storage of activations
 * and weights with fp32 accumulation. */
enum { ILLUMINA_PRECISION_F32 = 0, ILLUMINA_PRECISION_BF16 = 1 };

/* Frame layouts accepted by the forward pass. Components in [0, 1]. */
enum {
  ILLUMINA_FRAME_RGB_PLANAR = 0,     /* N x 3 x S x S float32  */
  ILLUMINA_FRAME_RGBA_INTERLEAVED = 1 /* N x S x S x 4 float32, alpha ignored */
};

/* Last error message of this thread ("" when none). */
const char *illumina_last_error(void);
/* Library version string. */
const char *illumina_version(void);
/* Number of CUDA devices visible to the library (0 without a GPU). */
int illumina_device_count(void);

/* ---------------------------------------------------------------------------
 * Layer table, weights, arena (pure host logic; no GPU needed)
 * ------------------------------------------------------------------------- */

/* buildArchitecture + costOf + weightSpecs (src/model/arch.ts:191-489,
 * src/model/weights.ts:29-63) as one JSON document:
 * {"name","inputSize","mean","std","tensors":{name:[h,w,c]},"ops":[...],
 *  "cost":[{"name","kind","macs","params"}],"totalMacs","totalParams",
 *  "specs":[[name,[shape]]]}. Writes at most `cap` bytes (NUL-terminated) and
 * stores the required size (including the NUL) in *needed. */
illumina_status illumina_arch_json(int input_size, char *buf, size_t cap, size_t *needed);

/* planArena + validateArena (src/engine/arena.ts:57-172) with the runner's
 * exclusion of the `depth` tensor (src/model/runner.ts:190-192), as JSON:
 * {"bufferSizes":[vec4 counts],"assignment":{name:index},"totalBytes","naiveBytes"}. */
illumina_status illumina_arena_json(int input_size, char *buf, size_t cap, size_t *needed);

/* Total float count of the weight blob (all tensors of weightSpecs, in order). */
illumina_status illumina_weights_count(int input_size, size_t *count);

/* synthesizeWeights(arch, seed) (src/model/weights.ts:227-251) into a flat
 * float blob in weightSpecs order. */
illumina_status illumina_weights_synthesize(int input_size, uint32_t seed, float *out, size_t count);

/* parseWeights (src/model/weights.ts:97-165): validates an idm/1 container
 * (f32 or f16 tensors) and writes the flat blob in weightSpecs order.
 * Errors: ILLUMINA_BAD_WEIGHTS or ILLUMINA_ARCH_MISMATCH with the reference's
 * messages. */
illumina_status illumina_weights_parse(int input_size, const void *bytes, size_t len, float *out,
                                       size_t count);

/* serializeWeights (src/model/weights.ts:168-194): flat blob -> idm/1 bytes
 * (compact JSON header, f32 tensors). *needed receives the byte size. */
illumina_status illumina_weights_serialize(int input_size, const float *blob, size_t count, void *out,
                                           size_t cap, size_t *needed);

/* halfToFloat (src/model/weights.ts:82-95). */
double illumina_half_to_float(uint16_t h);

/* ---------------------------------------------------------------------------
 * Depth model (createDepthModel / DepthModel, src/model/runner.ts:79-485)
 * ------------------------------------------------------------------------- */

typedef struct illumina_model illumina_model;

typedef struct illumina_model_options {
  int input_size;          /* network resolution, multiple of 32 (arch.ts:191) */
  int device;              /* CUDA device ordinal */
  int max_batch;           /* largest frame count per forward call */
  int precision;           /* ILLUMINA_PRECISION_* */
  int decode_srgb;         /* DepthModelOptions.decodeSrgb (runner.ts:90-91) */
  float exposure;          /* DepthModelOptions.exposure (runner.ts:92) */
  float range_sigma;       /* DepthPostParams x (runner.ts:185-187), 0.12 */
  float temporal_base;     /* DepthPostParams y, 0.35 */
  float temporal_sensitivity; /* DepthPostParams z, 3.0 */
  int keep_intermediates;  /* 1: no arena aliasing, every tensor stays readable */
  /* Weights, first non-empty source wins: flat blob, .idm bytes, .idm path,
   * else synthesizeWeights(arch, synth_seed) (the app's fallback, main.ts:61). */
  const float *weights;
  size_t weights_count;
  const void *idm_bytes;
  size_t idm_len;
  const char *idm_path;
  uint32_t synth_seed;
  int gemm_engine;         /* ILLUMINA_ENGINE_* for the pw / dw->pw / lateral ops */
} illumina_model_options;

/* Engines for the pointwise-shaped ops: tcgen05 tensor cores with TMEM
 * accumulators (fp32 storage: 3xTF32 split products; bf16: kind::f16), or the
 * CUDA-core register-blocked tile GEMM. */
enum { ILLUMINA_ENGINE_TENSOR = 0, ILLUMINA_ENGINE_SIMT = 1 };

/* Defaults: 448, device 0, batch 1, fp32, sRGB on, exposure 1, (0.12, 0.35,
 * 3.0), aliased arena, synthetic seed 1. */
void illumina_model_options_default(illumina_model_options *opts);

/* createDepthModel (runner.ts:160-485): parses/validates weights, plans and
 * validates the arena, uploads and packs weights once, allocates one device
 * arena sized for max_batch. Nothing is allocated per forward afterwards. */
illumina_status illumina_model_create(const illumina_model_options *opts, illumina_model **out);
/* DepthModel.destroy (runner.ts:478-484). */
illumina_status illumina_model_destroy(illumina_model *model);
/* DepthModel.setExposure (runner.ts:456-460). */
illumina_status illumina_model_set_exposure(illumina_model *model, float exposure);
/* DepthModel.setTemporal (runner.ts:461-465). */
illumina_status illumina_model_set_temporal(illumina_model *model, float base_alpha,
                                            float motion_sensitivity, float range_sigma);

/* The whole hot path for n independent frames (first-frame temporal
 * semantics, io.ts:259-266): preprocess -> 38 convolutions -> head ->
 * bilateralUp. `disparity` receives n x S x S float32 (the `depth` texture's
 * x channel); `depth_low` (nullable) receives n x S/2 x S/2 float32 (head
 * output, channel 0). The launch sequence is captured once per distinct
 * (n, pointers) and replayed as a CUDA graph.
 * ILLUMINA_TIMEOUT: a tensor-core kernel gave up a bounded wait (its outputs
 * are undefined; the model stays usable). A call with a host buffer
 * synchronises and reports its own kernels; a call on device buffers only
 * queues them, and a give-up is reported by the model's next forward, record
 * or illumina_model_sync (the reference's device errors are asynchronous
 * too: uncaptured-error events, src/main.ts). */
illumina_status illumina_forward(illumina_model *model, const float *frames, int n, int frame_layout,
                                 float *disparity, float *depth_low, void *stream);

/* The hot path from 8-bit RGBA source images, the reference's frame path: a
 * camera or canvas frame uploaded as an rgba8unorm texture (src/main.ts,
 * src/scene/blit.ts) and read by makePreprocess (kernels/io.ts:64-118).
 * `rgba8`: n images of src_h x src_w x 4 bytes, host or device, 4-byte
 * aligned; sampled as illumina_sample_source does (uv_scale / uv_offset
 * nullable: (1,1) / (0,0); `mirror` flips u), then illumina_forward on the
 * sampled planar frames. `disparity` (host, device or NULL) receives
 * n x S x S float32. With host buffers the call is synchronous and runs in
 * frame chunks whose uploads, sampling, graphs and downloads overlap; a host
 * source moves 4 bytes per source pixel over PCIe, against 12 per network
 * pixel for planar float frames. A host source larger than the model's
 * staging room (max_batch x S x S x 4 bytes) is staged in a device buffer the
 * model allocates on first need. ILLUMINA_TIMEOUT as for illumina_forward. */
illumina_status illumina_forward_source(illumina_model *model, const uint8_t *rgba8, int n, int src_w, int src_h,
                                        const float *uv_scale, const float *uv_offset, int mirror, float *disparity,
                                        void *stream);

/* The forward as the reference issues frames (one queue.submit per frame, no
 * fences, src/engine/frame.ts:1-19; readbacks awaited asynchronously,
 * src/main.ts:572-573) for pinned host
 * buffers: queues the upload of `frames` (n frames, `frame_layout`), the
 * forward of the whole batch as one graph and the download of the disparity
 * (n x S x S float32) into `disparity`, and returns. Both buffers must be
 * pinned host memory (cudaHostAlloc / cudaHostRegister) and stay untouched
 * until the work is done: illumina_model_sync waits for everything queued on
 * the model; `stream` (nullable) is made to wait for this call's download
 * (the upload does not wait for `stream`: the frames are host memory).
 * Consecutive calls alternate two device staging slots (allocated on the first
 * call, 2 x max_batch x S x S x 5 floats), so one call's transfers overlap the
 * neighbouring calls' graphs. ILLUMINA_TIMEOUT as for illumina_forward, reported
 * by the next call or illumina_model_sync. */
illumina_status illumina_forward_async(illumina_model *model, const float *frames, int n, int frame_layout,
                                       float *disparity, void *stream);

/* illumina_forward_async for 8-bit RGBA source images: `rgba8` (pinned host,
 * n images of src_h x src_w x 4 bytes, 4-byte aligned) is uploaded, sampled
 * as illumina_sample_source does and forwarded; the disparity (pinned host,
 * n x S x S float32) comes back asynchronously. Sources of up to S x S pixels
 * are staged in the asynchronous slots; larger ones in two source buffers the
 * model allocates (or grows, after waiting for its queued work) on need. */
illumina_status illumina_forward_source_async(illumina_model *model, const uint8_t *rgba8, int n, int src_w,
                                              int src_h, const float *uv_scale, const float *uv_offset, int mirror,
                                              float *disparity, void *stream);

/* forwardReference from a given network input (scripts/ref-forward.ts:296-300,
 * an "input" bundle; src/model/reference.ts:360-451): `input` holds n x S x S x 4
 * float32 channels-last preprocess outputs (host or device). Runs the stem as
 * its own launch and the rest of the hot path; the bilateral guide is the
 * input's channel 3 (the unnormalised luminance). fp32 models only.
 * Synchronous; the intermediates are readable with debugTensor afterwards. */
illumina_status illumina_forward_input(illumina_model *model, const float *input, int n, float *disparity,
                                       float *depth_low);

/* DepthModel.record for one streaming frame (runner.ts:440-449): like
 * illumina_forward with n = 1, but the bilateral upsample blends with the
 * temporal history held in the model's depth ping-pong and writes the depth
 * texture (stabilised, raw, change, 1) into slot outputParity(). */
illumina_status illumina_model_record(illumina_model *model, const float *frame, int frame_layout,
                                      void *stream);
/* Waits for the work queued on the model's stream and reports a kernel that
 * gave up a bounded wait as ILLUMINA_TIMEOUT -- the synchronous check of a
 * device-buffer forward (the reference's `device.queue.onSubmittedWorkDone()`
 * plus its error scope, src/model/runner.ts:425-434). */
illumina_status illumina_model_sync(illumina_model *model);
/* Cycles a tensor-core pipeline wait may take before the kernel gives up and
 * reports ILLUMINA_TIMEOUT (0 = the default, ~1 s; the waits with which a
 * kernel that gave up drains its own copies and MMAs keep the default). A
 * fault-handling hook with no reference counterpart: a small limit makes a
 * forward's waits give up so that the error path can be exercised. Drops the
 * captured graphs. */
illumina_status illumina_model_set_wait_limit(illumina_model *model, long long cycles);
/* DepthModel.swapHistory / outputParity / freshParity (runner.ts:450-454). */
illumina_status illumina_model_swap_history(illumina_model *model);
int illumina_model_output_parity(const illumina_model *model);
int illumina_model_fresh_parity(const illumina_model *model);
/* DepthModel.debugDepth (runner.ts:455): device pointer of depth slot `index`
 * (S x S x 4 float32: stabilised, raw, change, validity). */
illumina_status illumina_model_depth_slot(illumina_model *model, int index, const float **device_ptr);

/* DepthModel.debugTensor (runner.ts:466-476): copies frame 0 of tensor `name`
 * (h x w x c float32, channels-last) into `out` (host or device, at most
 * `cap` floats) and reports whether the tensor still owns its arena buffer
 * after a full forward (live_at_end = 0 when a later tensor reused it). */
illumina_status illumina_model_debug_tensor(illumina_model *model, const char *name, float *out,
                                            size_t cap, int *h, int *w, int *c, int *live_at_end);

/* DepthModel.debugTensor (runner.ts:466-476) for frame `frame` (0 <= frame <
 * max_batch) of the last batched forward; illumina_model_debug_tensor is this
 * call with frame 0. INVALID_ARG for a frame outside the model's batch. The
 * name "scene_color" reads the preprocess's second output (S x S x 4 linear
 * colour, alpha 1; ref-forward.ts:286-292), which a keep-intermediates model
 * keeps. */
illumina_status illumina_model_debug_tensor_frame(illumina_model *model, const char *name, int frame, float *out,
                                                  size_t cap, int *h, int *w, int *c, int *live_at_end);

/* DepthModel.stats (runner.ts:95-101, :425-434). */
typedef struct illumina_stats {
  int dispatches;          /* ops in the layer table (40) */
  int launches;            /* kernels one forward launches */
  size_t arena_bytes;      /* aliased activation bytes per frame (fp32 accounting) */
  size_t naive_arena_bytes;/* one buffer per tensor, per frame */
  size_t weight_bytes;     /* logical weight bytes (fp32) */
  size_t device_bytes;     /* device memory the model holds */
  int max_batch;
  int precision;
  int input_size;
  int gemm_engine;         /* ILLUMINA_ENGINE_* */
  int device_error;        /* non-zero: a kernel gave up a bounded wait (reads a device flag; synchronises) */
} illumina_stats;
illumina_status illumina_model_stats(const illumina_model *model, illumina_stats *out);

/* GpuProfiler analogue (src/engine/timing.ts:48-191): runs the op list
 * `reps` times as individual launches on the model's stream with a CUDA event
 * between consecutive ops, and writes the mean device time of each op in
 * milliseconds to op_ms[0..40) (an op fused into its neighbour reports 0).
 * `frames` must be device memory. For profiling only; the forward path
 * replays the captured graph instead. */
illumina_status illumina_model_profile(illumina_model *model, const float *frames, int n, int frame_layout,
                                       int reps, float *op_ms, int cap);

/* ---------------------------------------------------------------------------
 * Per-kernel entry points (the kernel factories under src/model/kernels/).
 * All pointers are device pointers; weights are in the logical .idm layout.
 * ------------------------------------------------------------------------- */

/* Selects, for the calling thread, the engine the per-kernel entry points
 * below use for pointwise / dw->pw / lateral (ILLUMINA_ENGINE_*; default
 * SIMT). No reference counterpart: the reference has one WGSL kernel per op. */
illumina_status illumina_set_op_engine(int engine);

/* makePointwise (kernels/pointwise.ts:64-133): dst[p][oc] = act(b[oc] +
 * sum_ic w[oc][ic]*src[p][ic] (+ res[p][oc])). */
illumina_status illumina_op_pointwise(const float *src, long pixels, int in_c, const float *w,
                                      const float *b, int out_c, int act, const float *res, float *dst,
                                      void *stream);

/* makeDepthwisePointwise (kernels/dwpw.ts:165-296): depthwise k x k stride s
 * (+dw_b, mid_act) then 1x1 (+pw_b, +res, act). dw_w is [in_c][k][k]. */
illumina_status illumina_op_dwpw(const float *src, int in_h, int in_w, int in_c, const float *dw_w,
                                 const float *dw_b, int mid_act, const float *pw_w, const float *pw_b,
                                 int out_c, int k, int stride, int act, const float *res, float *dst,
                                 void *stream);

/* The fused depthwise -> pointwise op of illumina_op_dwpw, for callers that
 * cannot allocate device memory. It has no counterpart in the reference.
 *
 * Why: illumina_op_dwpw obtains a temporary buffer (cudaMallocAsync) to
 * repack the depthwise weights. Some callers cannot allow that: a real-time
 * frame loop with a fixed device-memory budget, where an allocation may fail
 * or wait for memory mid-frame; or a host application whose own memory
 * manager reserves the device heap up front and forbids plugins from
 * allocating. This variant repacks into a fixed device array compiled into the
 * library (ILLUMINA_NOALLOC_DW_MAX_FLOATS floats, 256 KiB, reserved on every
 * GPU that loads the library until the process exits) and calls no
 * allocation routine.
 *
 * Limit: in_c * k * k must not exceed ILLUMINA_NOALLOC_DW_MAX_FLOATS, else the
 * call returns ILLUMINA_INVALID_ARG. The first call on a device resolves the
 * array's device address (cudaGetSymbolAddress) with that device current; make
 * that first call before any stream capture. All calls share the array: calls
 * whose GPU work overlaps (other streams or host threads on the same device)
 * race. Arguments and result are those of illumina_op_dwpw; the work runs on
 * the SIMT engine whatever illumina_set_op_engine selected for the calling
 * thread (the tensor engine's weight images would need an allocation). */
#define ILLUMINA_NOALLOC_DW_MAX_FLOATS 65536
illumina_status illumina_op_dwpw_noalloc(const float *src, int in_h, int in_w, int in_c, const float *dw_w,
                                         const float *dw_b, int mid_act, const float *pw_w, const float *pw_b,
                                         int out_c, int k, int stride, int act, const float *res, float *dst,
                                         void *stream);

/* makeConv (kernels/conv.ts:94-168): dense k x k stride s, zero pad, w is
 * [out_c][in_c][k][k]. */
illumina_status illumina_op_conv(const float *src, int in_h, int in_w, int in_c, const float *w,
                                 const float *b, int out_c, int k, int stride, int act, float *dst,
                                 void *stream);

/* makeLateral (kernels/lateral.ts:46-169): act(b + up2(coarse) + W skip);
 * coarse is ch x cw x out_c, skip is 2ch x 2cw x skip_c, w is [out_c][skip_c]. */
illumina_status illumina_op_lateral(const float *coarse, int ch, int cw, const float *skip, int skip_c,
                                    const float *w, const float *b, int out_c, int act, float *dst,
                                    void *stream);

/* makeHead (kernels/io.ts:141-166): dst4[p] = sigmoid(b + w.src[p]) x 4. */
illumina_status illumina_op_head(const float *src, long pixels, int in_c, const float *w, float b,
                                 float *dst4, void *stream);

/* makePreprocess (kernels/io.ts:64-118) for a source already at network
 * resolution: frames (layout as above) -> input tensor (S x S x 4) and
 * sceneColor (S x S x 4, nullable). */
illumina_status illumina_op_preprocess(const float *frames, int n, int frame_layout, int size,
                                       int decode_srgb, float exposure, float *input, float *scene_color,
                                       void *stream);

/* makeDepthUpsample (kernels/io.ts:203-283), first frame: low is lh x lw x
 * low_c (channel 0 read), guide is (2lh) x (2lw) x guide_c linear colour,
 * dst is (2lh) x (2lw) float32. */
illumina_status illumina_op_bilateral(const float *low, int lh, int lw, int low_c, const float *guide,
                                      int guide_c, float range_sigma, float *dst, void *stream);

/* ---------------------------------------------------------------------------
 * Lighting (src/lighting/)
 * ------------------------------------------------------------------------- */

#define ILLUMINA_MAX_LIGHTS 8 /* lights.ts:147 */

/* Light struct, field for field (lights.ts:132-144). */
typedef struct illumina_light {
  float position[4];  /* xyz view-space position (direction for directional) */
  float color[4];     /* rgb linear colour, a = intensity (0 = slot unused) */
  float direction[4]; /* xyz spot axis, w = cos(outer cone) */
  float params[4];    /* x kind (0 point, 1 spot, 2 directional), y cos(inner), z radius, w shadow */
} illumina_light;

/* ShadingSettings, field for field (renderer.ts:53-78). */
typedef struct illumina_shading_settings {
  float fov_y, near_m, far_m;
  float ao_strength, shadow_strength, volumetric, exposure;
  float ambient[3];
  float ambient_intensity, roughness, fog_density;
  float fog_color[3];
  float specular, normal_strength, albedo_mix, contact_shadow_length, ao_radius_pixels;
  int tone_map; /* 0 ACES fitted, 1 Reinhard */
  float contrast, saturation, vignette;
  int debug_view; /* 0 lit, 1 depth, 2 normals, 3 occlusion, 4 albedo */
} illumina_shading_settings;

/* DEFAULT_SETTINGS (renderer.ts:80-103). */
void illumina_shading_settings_default(illumina_shading_settings *s);

/* March step counts. The reference compiles contact 12 (shade.ts:192), AO
 * 6 directions x 4 steps (:232-233) and 10 volumetric steps per light (:310). */
typedef struct illumina_shade_steps {
  int contact, ao_dirs, ao_steps, volumetric;
} illumina_shade_steps;

/* makeShade + composite (shade.ts:312-528, composite.ts:87-113) in one pass:
 * disparity is dh x dw texels of `disparity_channels` float32 each (channel 0
 * read, nearest fetch; 4 reads a depth slot directly), albedo is a 3 x ah x aw
 * sRGB image (bilinear, clamp-to-edge), lights is ILLUMINA_MAX_LIGHTS slots.
 * `steps` NULL selects the reference's constants. Outputs (either nullable):
 * hdr (out_h x out_w x 4 float32, the HDR target) and rgba8 (out_h x out_w x 4
 * bytes, tone-mapped 8-bit sRGB). Device pointers only. */
illumina_status illumina_shade(const float *disparity, int dw, int dh, int disparity_channels,
                               const float *albedo, int aw,
                               int ah, const illumina_light *lights,
                               const illumina_shading_settings *settings, uint32_t frame,
                               const illumina_shade_steps *steps, int out_w, int out_h, float *hdr,
                               uint8_t *rgba8, void *stream);

/* Bilinear resize of a single-channel map (align_corners=false, edge clamp),
 * used to bring the disparity to render resolution. Device pointers. */
illumina_status illumina_resize_bilinear(const float *src, int sw, int sh, float *dst, int dw, int dh,
                                         void *stream);

/* The source-texture read of makePreprocess (kernels/io.ts:64-118) for an
 * 8-bit RGBA source of any size: n images of src_h x src_w x 4 bytes (device)
 * are sampled at uv = ((x+0.5)/size, (y+0.5)/size) * uv_scale + uv_offset
 * (createDepthModel's uvScale/uvOffset, runner.ts:88-89, :181-182; NULL means
 * (1,1) and (0,0)), u mirrored first when `mirror` (the blit's mirror,
 * scene/blit.ts:57-60), with linear filtering and clamp-to-edge
 * (runner.ts:177), texels read as value/255. Output: n x 3 x size x size
 * planar float frames for illumina_forward (FRAME_RGB_PLANAR), which applies
 * the sRGB decode, exposure and normalisation. */
illumina_status illumina_sample_source(const uint8_t *rgba8, int n, int src_w, int src_h, const float *uv_scale,
                                       const float *uv_offset, int mirror, int size, float *frames,
                                       void *stream);

/* cropTransform (scene/blit.ts:80-86): the largest centred square of a
 * width x height image as {scaleX, scaleY, offsetX, offsetY}, for
 * illumina_sample_source's uv_scale = out[0..1], uv_offset = out[2..3]. */
void illumina_crop_transform(int width, int height, float out[4]);

/* ---------------------------------------------------------------------------
 * Procedural scene and depth metrics (src/scene/)
 * ------------------------------------------------------------------------- */

/* SceneParams (procedural.ts:23-30): camera = xyz position + time in seconds,
 * focus = xyz look-at point + tan(fovY/2), options = aspect, far plane,
 * key-light azimuth, scene variant. */
typedef struct illumina_scene_params {
  float camera[4];
  float focus[4];
  float options[4];
} illumina_scene_params;

/* The uniforms createProceduralScene starts with (procedural.ts:295-299). */
void illumina_scene_params_initial(illumina_scene_params *p);

/* ProceduralScene.update(time, orbit) (procedural.ts:310-318): the camera
 * orbit and the key light's drift, evaluated in double and stored as float. */
void illumina_scene_params_update(illumina_scene_params *p, double time_seconds, int orbit);

/* The ray-marched SDF scene (sceneVertex/sceneFragment, procedural.ts:177-273)
 * for n frames of width x height, frame i with params[i] (host array). It
 * replaces the record() draw into an rgba8unorm colour target and an
 * rgba16float truth target with device buffers, each nullable:
 *   rgb   n x 3 x height x width float32: the 8-bit colour as value/255, the
 *         planar frame layout illumina_forward takes (what sampling the
 *         rgba8unorm source texture yields);
 *   rgba8 n x height x width x 4 bytes: the colour target itself;
 *   truth n x height x width x 2 float32: (distance along the view axis, hit
 *         mask), the truth target's x and y, kept in float32.
 * Pixel (x, y), y down, is the fragment at uv = ((x+0.5)/width, (y+0.5)/height). */
illumina_status illumina_scene_render(const illumina_scene_params *params, int n, int width, int height,
                                      float *rgb, uint8_t *rgba8, float *truth, void *stream);

/* DepthMetrics (metrics.ts:17-32). */
typedef struct illumina_depth_metrics {
  long long samples;
  double abs_rel, rmse, delta1, delta2, delta3, scale, shift;
} illumina_depth_metrics;

/* evaluateDepth (metrics.ts:66-161) for n frames on the device, without the
 * reference's texture readback: predicted disparity is channel 0 of
 * pred_channels-float texels (1 for illumina_forward's disparity, 4 for a
 * depth slot), truth is the scene's (depth, hit) pairs, both width x height per
 * frame. Least-squares scale/shift in disparity space over pixels with hit >=
 * 0.5 and 0.05 < depth <= 25, then AbsRel, RMSE and delta1..3 of the aligned
 * depth, in double; fewer than 64 valid pixels gives NaN errors and zero
 * deltas, as the reference does. out: n structs, device memory. */
illumina_status illumina_evaluate_depth(const float *pred, int pred_channels, const float *truth, int n, int width,
                                        int height, illumina_depth_metrics *out, void *stream);

/* ---------------------------------------------------------------------------
 * Synthetic workloads and checksums
 * ------------------------------------------------------------------------- */

enum { ILLUMINA_FRAMES_UNIFORM = 0, ILLUMINA_FRAMES_BLOBS = 1 };

/* Seeded frames on the device, 3 x size x size planar each; frame i uses seed
 * seed0 + i. UNIFORM: float32 of mulberry32 draws in (c, y, x) order. BLOBS:
 * 8 anisotropic Gaussian blobs per channel + N(0, 0.02) noise, clamped. */
illumina_status illumina_generate_frames(int kind, uint32_t seed0, int n, int size, float *out,
                                         void *stream);

/* Per-frame checksums of n maps of `count` float32 each (device pointer):
 * sum64[i] = sum_j bits(x_j) * (2j + 1) mod 2^64 and fsum[i] = sum_j x_j
 * (double). Outputs are device pointers. */
illumina_status illumina_checksums(const float *maps, int n, long count, uint64_t *sum64, double *fsum,
                                   void *stream);

/* Exhaustive device check of an arithmetic helper of the tensor-core kernels
 * against the operation it replaces, over all 2^32 binary32 bit patterns
 * except NaNs: which = 0 the TF32 rounding of the 3xTF32 hi/lo split against
 * cvt.rna.tf32.f32, which = 1 the division by 6 of hardswish against the IEEE
 * quotient. result (host, 3 values): inputs checked, mismatches, and the bits
 * of one mismatching input (all ones when there is none). Runs on the current
 * device, synchronously. No counterpart in the reference. */
illumina_status illumina_selftest(int which, unsigned long long *result);

#ifdef __cplusplus
}
#endif

#endif /* ILLUMINA_H */
