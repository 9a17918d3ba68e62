/*
 * rechead.h — C ABI of the B200-native (sm_100a) quantised recognition head of
 * rust-ppocrv6: the per-class symmetric INT8 W8A32 projection of SVTR features onto the CTC
 * vocabulary (graph node MatMul.12 with the folded bias Add.204), softmax (Softmax.2) and
 * the per-timestep greedy argmax that CTC decoding consumes.
 *
 * Every entry point replaces one call the Rust engine makes today; each declaration cites
 * the reference item it stands in for (paths inside the rust-ppocrv6 project).
 *
 * Conventions
 *  - Plain pointers and sizes; no ownership passes except through the opaque handles.
 *  - Functions return RH_OK (0) or an RH_ERR_* code. rh_last_error() then describes the
 *    failure of the calling thread's most recent call. RH_ERR_INVALID_ARG is the analogue of
 *    the reference's OcrError::OperatorError (src/error.rs:4-27); nothing here aborts the
 *    process (the reference keeps panic = "abort" off for embedders, Cargo.toml:41-45).
 *  - "Host" entry points take host memory (pinned or pageable) and return when the results
 *    are in host memory. "_device" entry points take device memory of one context device
 *    and a cudaStream_t (as void*), enqueue asynchronously and report device-side failures
 *    at the next rh_sync() on that device.
 *  - Requires an sm_100 (B200-class) GPU. There is no CPU fallback: rh_ctx_create fails
 *    with RH_ERR_NO_DEVICE / RH_ERR_UNSUPPORTED when no such device is present.
 *  - Calls on one context are serialised per device and are safe from many threads (the
 *    engine calls the head from up to rec_batch_threads Rayon workers, src/pipeline.rs:417-427).
 */
#ifndef RECHEAD_H
#define RECHEAD_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RH_OK 0
#define RH_ERR_INVALID_ARG 1  /* bad shape, length or pointer: OcrError::OperatorError */
#define RH_ERR_CUDA 2         /* a CUDA runtime call failed */
#define RH_ERR_TIMEOUT 3      /* a kernel's bounded wait ran out; the context stays usable */
#define RH_ERR_UNSUPPORTED 4  /* K > 128, or a device that is not sm_100 */
#define RH_ERR_NO_DEVICE 5    /* no CUDA device */
#define RH_ERR_DEVICE_FAULT 6 /* a device shard failed and no healthy device could redo it */

typedef struct rh_ctx rh_ctx;
typedef struct rh_weight rh_weight;

/* Library version (major * 10000 + minor * 100 + patch). */
int rh_version(void);

/* Number of visible CUDA devices. */
int rh_device_count(int *count);

/* Message for the calling thread's most recent failed call ("" if none). Never NULL. */
const char *rh_last_error(void);

/*
 * Creates a context over `n_devices` CUDA devices (devices == NULL: device 0 only). Each
 * device gets its own stream, status word and scratch. Batched host calls shard their lines
 * over these devices. Replaces the engine's recognition worker pool for this head
 * (OcrEngine::with_config rec_pool, src/pipeline.rs:232-251).
 */
int rh_ctx_create(const int *devices, int n_devices, rh_ctx **out);
void rh_ctx_destroy(rh_ctx *ctx);
int rh_ctx_num_devices(const rh_ctx *ctx);
/* Upper bound on any device-side wait, in milliseconds (default 2000). */
int rh_ctx_set_timeout_ms(rh_ctx *ctx, int timeout_ms);

/*
 * Quantises and packs the transposed head weight w_nk [n][k] (row j = class j, as built by
 * the load-time transpose in src/engine/model.rs:565-605) on every context device, with the
 * bias folded in (bias may be NULL; otherwise bias_len must equal n, as
 * src/ops/matmul.rs:1288-1295 requires). Bit-exact with QuantizedWeight::from_f32_transposed
 * (src/ops/matmul.rs:1173-1202) as called by Model::quantize_matmul_weights
 * (src/engine/model.rs:628-638) when OcrEngineConfig.quantize_rec_head is set
 * (src/pipeline.rs:197-199). Keeps no host copy of the FP32 weight. 1 <= k <= 128.
 */
int rh_weight_pack(rh_ctx *ctx, const float *w_nk, int64_t n, int64_t k, const float *bias, int64_t bias_len,
                   rh_weight **out);

/*
 * rh_weight_pack with the weight kept in HBM as int8 (16 KB per 128 classes, q + 128 per byte,
 * plus the f32 (scale, bias) table): 2.56 MB for the 18710 x 120 head, against 8.98 MB for the
 * FP32 copy, the footprint cut of Model::quantize_matmul_weights that the reference asserts
 * (src/engine/model.rs:2905-2920: at least 3.5x). The kernel expands each tile to fp16 in shared
 * memory, which costs issue slots: decoded results are bit-identical to rh_weight_pack's, at
 * lower throughput. Same arguments and errors as rh_weight_pack.
 */
int rh_weight_pack_compact(rh_ctx *ctx, const float *w_nk, int64_t n, int64_t k, const float *bias,
                           int64_t bias_len, rh_weight **out);

/* Replaces the folded bias (NULL: no bias). bias_len must equal n. The MatMul arm passes the
 * folded Add.204 bias on every call (src/engine/model.rs:1248-1252, :1261-1262). */
int rh_weight_set_bias(rh_ctx *ctx, rh_weight *w, const float *bias, int64_t bias_len);

/* Copies out QuantizedWeight::data (int8 [n][k]) and ::scales (f32 [n]) from the first
 * context device (src/ops/matmul.rs:1165-1171); either pointer may be NULL. */
int rh_weight_export(rh_ctx *ctx, const rh_weight *w, int8_t *q, float *scales);

/* Copies out the device form of a quantised weight: its tiles (n_chunks = ceil(n/128) tiles of
 * rh_weight_tile_bytes bytes) and its class table (n_chunks * 256 floats: per tile scale[128],
 * then bias[128]; padded classes (0, -inf)). Either pointer may be NULL. Tile t holds classes
 * 128 t .. 128 t + 127 (row r = class - 128 t) over K slots s < 128:
 *  - rh_weight_pack: fp16 q at byte (s / 64) 16384 + 128 r + 16 (((s % 64) / 8) ^ (r % 8)) + 2 (s % 8)
 *    (the tensor core's 128-byte-swizzled operand image);
 *  - rh_weight_pack_compact: byte q + 128 at 16 ((8 (r / 8) + s / 16) 8 + r % 8) + s % 16.
 * K slots >= k hold q = 0, except that when the last 16-slot step holds <= 8 values its upper 8
 * slots repeat the lower 8. */
int rh_weight_export_image(rh_ctx *ctx, const rh_weight *w, uint8_t *tiles, float *table);

/* Bytes per 128-class tile of the packed weight on the device: 32768 (rh_weight_pack), 16384
 * (rh_weight_pack_compact), 65536 (rh_weight_pack_f32); 0 for NULL. */
int64_t rh_weight_tile_bytes(const rh_weight *w);

int rh_weight_dims(const rh_weight *w, int64_t *n, int64_t *k);

/* Device bytes held per device by the packed weight: its tiles plus the (scale, bias) class
 * table, nothing else (Model::weight_footprint_bytes, src/engine/model.rs:651-667, for the
 * head). 18710 x 120 head: 2,558,976 compact, 4,967,424 fp16 image, 9,784,320 FP32. */
int64_t rh_weight_device_bytes(const rh_weight *w);

void rh_weight_free(rh_weight *w);

/*
 * out[r][j] = (sum_i a[r][i] * q[j][i]) * scale[j] + bias[j] for r < rows, j < n: the
 * literal drop-in for matmul_quantized_b (src/ops/matmul.rs:1204-1336) as dispatched by
 * the MatMul arm for MatMul.12 (src/engine/model.rs:1245-1272). `k` must equal the
 * weight's K (the check at src/ops/matmul.rs:1227-1232). a is [rows][k], out [rows][n],
 * both host memory. rows == 0 is a no-op.
 */
int rh_matmul_quantized_b(rh_ctx *ctx, const rh_weight *w, const float *a, int64_t rows, int64_t k, float *out);

/*
 * The FP32 head, the engine's default (OcrEngineConfig.quantize_rec_head is false by default,
 * src/pipeline.rs:59): the MatMul arm then runs matmul_transposed_b (src/ops/matmul.rs:514-897,
 * dispatched at src/engine/model.rs:1264) on the transposed FP32 weight. rh_weight_pack_f32
 * keeps no int8: each class row is scaled by an exact power of two and split into fp16 high
 * and low parts (~22 significant bits, A split likewise), so logits match the FP32 product to
 * within 1e-4. The returned weight works with rh_matmul_transposed_b (the literal MatMul.12
 * drop-in in FP32 mode), rh_head_decode[_lines|_device|_ctc] and the device forms;
 * rh_weight_export/_image and rh_matmul_quantized_b reject it (and rh_matmul_transposed_b
 * rejects an INT8 weight). Same arguments and errors as rh_weight_pack / rh_matmul_quantized_b.
 */
int rh_weight_pack_f32(rh_ctx *ctx, const float *w_nk, int64_t n, int64_t k, const float *bias, int64_t bias_len,
                       rh_weight **out);
int rh_matmul_transposed_b(rh_ctx *ctx, const rh_weight *w, const float *a, int64_t rows, int64_t k, float *out);

/*
 * The fused head: for each timestep row r of a [rows][k], the class with the largest
 * probability after softmax over all n classes (first index on ties) and that probability,
 * i.e. matmul_quantized_b -> softmax_inplace (src/ops/softmax.rs:199-285, dispatched by the
 * Softmax arm src/engine/model.rs:1286-1302) -> find_argmax (src/postprocess/ctc.rs:178-258)
 * as CtcDecoder::decode_batch applies it per timestep (src/postprocess/ctc.rs:144-149).
 * The [rows][n] logits never leave the GPU. Host memory; runs on the first device.
 */
int rh_head_decode(rh_ctx *ctx, const rh_weight *w, const float *a, int64_t rows, int64_t k, int32_t *idx,
                   float *prob);

/*
 * rh_head_decode over a batch of text lines packed densely: line l owns rows
 * [line_offsets[l], line_offsets[l+1]) of a. Lines are split into contiguous shards of
 * balanced timestep count, one per context device, run concurrently, and gathered into
 * idx/prob (no collective: only the per-row results come back). Replaces the per-line
 * Rayon fan-out of OcrEngine::recognize (src/pipeline.rs:395-436) for this head. A shard
 * whose device fails is redone on a healthy device; results do not depend on the device.
 */
int rh_head_decode_lines(rh_ctx *ctx, const rh_weight *w, const float *a, const int64_t *line_offsets,
                         int64_t n_lines, int64_t k, int32_t *idx, float *prob);

/*
 * rh_head_decode on the SVTR tail's own layout: x is [batch][k][t_len] (the [B, 120, 1, T]
 * output after Squeeze.7 and before Transpose.8, src/engine/model.rs:1325-1343, graph nodes
 * Squeeze.7/Transpose.8), so the transpose to [batch*t_len][k] rows that feeds MatMul.12 is
 * folded into the kernel's feature loads (each converter thread gathers its timestep row; a
 * warp reads 32 consecutive timesteps per feature, coalesced). idx/prob are [batch*t_len] in
 * (b, t) order, exactly what rh_head_decode returns for the transposed rows. Host memory, the
 * batch split into equal line shards over the context's devices (as rh_head_decode_lines);
 * the _device form takes device pointers and a stream.
 */
int rh_head_decode_kt(rh_ctx *ctx, const rh_weight *w, const float *x, int64_t batch, int64_t k, int64_t t_len,
                      int32_t *idx, float *prob);
int rh_head_decode_kt_device(rh_ctx *ctx, const rh_weight *w, int slot, const float *d_x, int64_t batch,
                             int64_t t_len, int32_t *d_idx, float *d_prob, void *stream);

/* Device-memory forms on context device `slot` (0-based) and `stream` (cudaStream_t, NULL =
 * the legacy default stream). Asynchronous; failures surface at rh_sync(). Calls on one slot
 * from different streams are ordered on the slot's scratch by an event, so they never race. */
int rh_head_decode_device(rh_ctx *ctx, const rh_weight *w, int slot, const float *d_a, int64_t rows, int32_t *d_idx,
                          float *d_prob, void *stream);
int rh_matmul_quantized_b_device(rh_ctx *ctx, const rh_weight *w, int slot, const float *d_a, int64_t rows,
                                 float *d_out, void *stream);

/*
 * rh_head_decode_device with no memory allocation. No counterpart in the reference: it
 * exists for callers that cannot allocate device memory while they run — a host that
 * reserves all GPU memory up front for its own allocator, or a latency-critical loop that
 * must not call cudaMalloc/cudaFree because both synchronise the device.
 * Its only scratch (the per-split partial rows that the class-range split writes and the
 * merge kernel reads) is a fixed 4 MiB array in the library's device image, so every GPU that
 * uses the library holds those 4 MiB until the process exits. Limit: at most 262,144
 * timestep rows per call (larger calls fail with RH_ERR_INVALID_ARG and launch nothing); only
 * the row blocks after the last full wave are split, so a call needs at most about one wave's
 * rows (148 x 128) of partial entries whatever its size.
 *  - The first call on a device resolves the array's device address (cudaGetSymbolAddress,
 *    which may load the library's device code); make that first call before any stream
 *    capture.
 *  - Every call on a device shares the one array and no part of it has to start at zero (the
 *    head kernel writes every entry the merge kernel reads), but calls whose work overlaps on
 *    the GPU (different streams, or different contexts on the same device) race on it: order
 *    them on one stream or with events.
 *  - Calls no cudaMalloc, cudaFree or other allocating routine; the context and the packed
 *    weight are created beforehand. Failures surface at rh_sync(), as for the other
 *    "_device" forms.
 */
int rh_head_decode_device_noalloc(rh_ctx *ctx, const rh_weight *w, int slot, const float *d_a, int64_t rows,
                                  int32_t *d_idx, float *d_prob, void *stream);

/* Waits for all work on device `slot` (slot < 0: every device) and reports device-side
 * failures (RH_ERR_TIMEOUT) recorded since the previous rh_sync. */
int rh_sync(rh_ctx *ctx, int slot);

/* Number of head-kernel launches (head + merge + pack) issued on `slot` since creation. */
int64_t rh_launch_count(const rh_ctx *ctx, int slot);

/*
 * CTC greedy collapse on per-timestep (idx, prob): the loop of CtcDecoder::decode_batch
 * (src/postprocess/ctc.rs:144-169). For line l (timesteps [line_offsets[l],
 * line_offsets[l+1])) emit idx[t] when idx[t] != 0 (blank) and idx[t] != idx[t-1] (repeat;
 * the previous index starts at 0 for each line). tokens receives the emitted class indices
 * of all lines back to back (capacity >= line_offsets[n_lines] - line_offsets[0]);
 * token_offsets[l]..token_offsets[l+1] delimit line l (n_lines + 1 entries); scores[l] is
 * the f32 mean of the emitted probabilities (0 when none). Returns the number of tokens, or
 * -1 on invalid arguments. Host-only; needs no device.
 */
int64_t rh_ctc_collapse(const int32_t *idx, const float *prob, const int64_t *line_offsets, int64_t n_lines,
                        int32_t *tokens, int64_t *token_offsets, float *scores);

/*
 * rh_ctc_collapse on the GPU, device memory, on context device `slot` and `stream`
 * (cudaStream_t, NULL = the legacy default stream): the same rule and the same outputs
 * (d_tokens back to back, d_token_offsets with n_lines + 1 entries starting at 0, d_scores
 * bit-identical to the host loop) for (d_idx, d_prob) that rh_head_decode_device left on
 * the device. Replaces the collapse loop of CtcDecoder::decode_batch
 * (src/postprocess/ctc.rs:144-169) after a GPU head. d_line_offsets index d_idx/d_prob
 * (non-decreasing; a decreasing pair counts as an empty line); d_tokens needs room for
 * d_line_offsets[n_lines] - d_line_offsets[0] entries. Asynchronous: three kernel launches.
 */
int rh_ctc_collapse_device(rh_ctx *ctx, int slot, const int32_t *d_idx, const float *d_prob,
                           const int64_t *d_line_offsets, int64_t n_lines, int32_t *d_tokens, int64_t *d_token_offsets,
                           float *d_scores, void *stream);

/*
 * The whole recognition head of a batch of text lines with the collapse on the GPU:
 * rh_head_decode_lines (sharded over the context's devices) followed by
 * rh_ctc_collapse_device on each shard, so only the collapsed tokens and one score per line
 * leave the GPUs. Outputs as rh_ctc_collapse (host memory; tokens needs room for
 * line_offsets[n_lines] - line_offsets[0] entries). Replaces the per-line
 * matmul_quantized_b -> softmax_inplace -> CtcDecoder::decode chain of
 * OcrEngine::recognize (src/pipeline.rs:364-436, src/postprocess/ctc.rs:103-175) for this
 * head; text = the vocabulary entries of the tokens (CtcDecoder::decode_indices in the
 * binding). Same errors as rh_head_decode_lines.
 */
int rh_head_decode_ctc(rh_ctx *ctx, const rh_weight *w, const float *a, const int64_t *line_offsets, int64_t n_lines,
                       int64_t k, int32_t *tokens, int64_t *token_offsets, float *scores);

/*
 * A padded batch end to end: the SVTR tail's [batch][k][t_len] output of a batch whose lines
 * were padded to one width (the packing of tools/profiling/batch_poc.rs:14-32), line b valid
 * for its first valid_t[b] timesteps (0 <= valid_t[b] <= t_len). The head runs on every
 * timestep as rh_head_decode_kt does (Transpose.8 folded into the loads), then the CTC collapse
 * of rh_ctc_collapse runs on the GPU over each line's valid timesteps only, which is what the
 * per-line chain of OcrEngine::recognize (src/pipeline.rs:364-436) decodes for that line.
 * Outputs as rh_ctc_collapse: tokens (room for sum(valid_t) entries), token_offsets
 * [batch + 1], scores [batch]; host memory, the batch split into equal line shards over the
 * context's devices (as rh_head_decode_ctc).
 */
int rh_head_decode_kt_ctc(rh_ctx *ctx, const rh_weight *w, const float *x, int64_t batch, int64_t k, int64_t t_len,
                          const int64_t *valid_t, int32_t *tokens, int64_t *token_offsets, float *scores);

/* ------------------------------------------------ batched recognition preprocessing
 *
 * The producer side of the head: text-line crops (RGB8, row-major HWC, 3 bytes per pixel)
 * into the recognition network's input tensor. Per crop this is RecPreprocess::process
 * (src/preprocess/rec.rs:60-105): width = clamp(ceil(H * w / max(h, 1)), 32, max(max_w, 32))
 * with H = max(target_h, 1); resize_exact(width, H, FilterType::Triangle) of the `image`
 * crate (0.25); v / 127.5 - 1 into channel planes. The batch is packed as the reference's
 * batching proof of concept packs it (tools/profiling/batch_poc.rs:14-32): out
 * [n_lines][3][H][wmax] f32, wmax = the largest width in the batch, columns past a line's
 * width = +1.0 (white). An empty crop (w or h == 0) resizes to black (-1.0).
 */

/* RecPreprocess::process's output width for one crop (src/preprocess/rec.rs:62-75).
 * Host only: needs no context or GPU. */
uint32_t rh_rec_resized_width(uint32_t orig_w, uint32_t orig_h, uint32_t target_h, uint32_t max_w);

/* Shape of a batch (host only): out_widths[n_lines] (may be NULL), H and wmax. Lets a caller
 * size the output of rh_rec_preprocess. RH_ERR_UNSUPPORTED for target_h > 2^20 or a crop
 * side > 2^30. */
int rh_rec_batch_shape(const uint32_t *widths, const uint32_t *heights, int64_t n_lines, uint32_t target_h,
                       uint32_t max_w, uint32_t *out_widths, uint32_t *out_h, uint32_t *out_wmax);

/*
 * Batched preprocessing from host memory, sharded over the context's devices (equal line
 * counts). Crop l is widths[l] x heights[l] pixels at byte rgb_offsets[l] of rgb[0, rgb_len).
 * out: host, >= n_lines * 3 * H * wmax floats (out_len); out_widths (may be NULL) and
 * *out_wmax (may be NULL) receive the batch shape. Replaces the per-crop loop
 * `self.rec_preprocess.process(&cropped_patch)` of OcrEngine::recognize
 * (src/pipeline.rs:379) plus build_batch. RH_ERR_INVALID_ARG: a crop outside the pixel
 * buffer, a short output; RH_ERR_UNSUPPORTED: a crop that shrinks by more than 6142x
 * horizontally (its filter window would not fit the kernel's shared-memory stage), sizes above
 * the limits of rh_rec_batch_shape.
 */
int rh_rec_preprocess(rh_ctx *ctx, const uint8_t *rgb, int64_t rgb_len, const int64_t *rgb_offsets,
                      const uint32_t *widths, const uint32_t *heights, int64_t n_lines, uint32_t target_h,
                      uint32_t max_w, float *out, int64_t out_len, uint32_t *out_widths, uint32_t *out_wmax);

/* As rh_rec_preprocess with the crops (d_rgb) and the output (d_out) in device memory of
 * `slot`'s device, enqueued on `stream` (0 = the legacy default stream); offsets and sizes
 * stay in host memory. Asynchronous: device-side errors surface at rh_sync. */
int rh_rec_preprocess_device(rh_ctx *ctx, int slot, const uint8_t *d_rgb, int64_t rgb_len, const int64_t *rgb_offsets,
                             const uint32_t *widths, const uint32_t *heights, int64_t n_lines, uint32_t target_h,
                             uint32_t max_w, float *d_out, int64_t out_len, uint32_t *out_widths, uint32_t *out_wmax,
                             void *stream);

#ifdef __cplusplus
}
#endif

#endif /* RECHEAD_H */
