/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of rust-ppocrv6's recognition preprocessing, batched:
 *   RecPreprocess::process   src/preprocess/rec.rs:60-105  (width rule, resize, normalise)
 *   build_batch              tools/profiling/batch_poc.rs:14-32  ([N,3,H,Wmax], +1.0 padding)
 * used by tests/ and bench.py's CPU legs as the CHECKER of the CUDA preprocessing kernels
 * and as their CPU baseline. The shipped library never links or loads this file.
 *
 * The resize itself lives in a third-party crate absent from the reference tree:
 * `image` 0.25.10 (Cargo.lock:1007-1010), called as
 * `img.resize_exact(target_w, target_h, FilterType::Triangle)` (rec.rs:77). Its published
 * algorithm is a separable filter: a vertical pass to f32 first, then a horizontal pass
 * that clamps to [0, 255] and rounds half away from zero. For each output coordinate o of
 * an axis of n_in -> n_out pixels: ratio = n_in / n_out, s = max(ratio, 1), the centre is
 * (o + 1/2) * ratio; the taps are the input pixels [floor(centre - s), ceil(centre + s))
 * clipped to the image (at least one); tap i weighs tri((i - (centre - 1/2)) / s) with
 * tri(x) = max(0, 1 - |x|), and the weights are divided by their f32 sum. Every sum runs
 * in tap order in f32, products are not fused (Rust never contracts a*b+c; this file is
 * built with -ffp-contract=off). An empty source image gives a zero (black) image.
 *
 * PARITY UNPINNED against the crate itself: its source is not in the reference tree and no
 * Rust toolchain exists here, so no output of the real resampler is available. The restated
 * algorithm is pinned against the reference's own rec.rs unit tests (output shapes, the
 * black-image values) and against properties any correct resampler has (identity when the
 * size does not change, solid colours stay solid).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_OK 0
#define OR_ERR_ARG 1

/* `v as u32` for f32: saturating, NaN -> 0. */
static uint32_t rust_f32_as_u32(float v) {
    if (!(v > 0.0f)) return 0;
    if (v >= 4294967296.0f) return UINT32_MAX;
    return (uint32_t)v;
}

/* Resized width of a crop: rec.rs:62-75 (target_h >= 1, max_w >= 32, aspect in f32,
 * ceil, saturating cast, clamp to [32, max_w]). */
uint32_t oracle_rec_resized_width(uint32_t orig_w, uint32_t orig_h, uint32_t target_h, uint32_t max_w) {
    const uint32_t h = orig_h > 1 ? orig_h : 1;
    const uint32_t th = target_h > 1 ? target_h : 1;
    const uint32_t mw = max_w > 32 ? max_w : 32;
    const float aspect = (float)orig_w / (float)h;
    uint32_t w = rust_f32_as_u32(ceilf((float)th * aspect));
    if (w < 32) w = 32;
    if (w > mw) w = mw;
    return w;
}

/* Tap window and normalised weights of output coordinate o (see the header). `wts` holds
 * at least ceil(2 s) + 3 floats. Returns the tap count; *left receives the first tap. */
static uint32_t tri_window(uint32_t n_in, uint32_t n_out, uint32_t o, float *wts, uint32_t *left) {
    const float ratio = (float)n_in / (float)n_out;
    const float s = ratio < 1.0f ? 1.0f : ratio;
    const float centre = ((float)o + 0.5f) * ratio;
    int64_t lo = (int64_t)floorf(centre - s);
    if (lo < 0) lo = 0;
    if (lo > (int64_t)n_in - 1) lo = (int64_t)n_in - 1;
    int64_t hi = (int64_t)ceilf(centre + s);
    if (hi < lo + 1) hi = lo + 1;
    if (hi > (int64_t)n_in) hi = (int64_t)n_in;
    const float c0 = centre - 0.5f;
    float sum = 0.0f;
    for (int64_t i = lo; i < hi; ++i) {
        const float x = fabsf(((float)i - c0) / s);
        const float w = x < 1.0f ? 1.0f - x : 0.0f;
        wts[i - lo] = w;
        sum += w;
    }
    for (int64_t j = 0; j < hi - lo; ++j) wts[j] /= sum;
    *left = (uint32_t)lo;
    return (uint32_t)(hi - lo);
}

static size_t tap_capacity(uint32_t n_in, uint32_t n_out) {
    const double r = (double)n_in / (double)n_out;
    return (size_t)ceil(2.0 * (r < 1.0 ? 1.0 : r)) + 3;
}

/* resize_exact(nw, nh, Triangle) of an RGB8 image (HWC, w x h) into dst (HWC, nw x nh). */
int oracle_resize_triangle_rgb8(const uint8_t *src, uint32_t w, uint32_t h, uint32_t nw, uint32_t nh,
                                uint8_t *dst) {
    if (nw == 0 || nh == 0) return OR_OK;
    if (w == 0 || h == 0) {
        memset(dst, 0, (size_t)nw * nh * 3);
        return OR_OK;
    }
    float *tmp = (float *)malloc((size_t)w * nh * 3 * sizeof(float));
    const size_t cap_y = tap_capacity(h, nh), cap_x = tap_capacity(w, nw);
    float *wts = (float *)malloc((cap_y > cap_x ? cap_y : cap_x) * sizeof(float));
    if (!tmp || !wts) {
        free(tmp);
        free(wts);
        return OR_ERR_ARG;
    }
    /* vertical pass: [h][w] u8 -> [nh][w] f32 */
    for (uint32_t oy = 0; oy < nh; ++oy) {
        uint32_t top;
        const uint32_t n = tri_window(h, nh, oy, wts, &top);
        for (uint32_t x = 0; x < w; ++x)
            for (int c = 0; c < 3; ++c) {
                float t = 0.0f;
                for (uint32_t j = 0; j < n; ++j) t += (float)src[((size_t)(top + j) * w + x) * 3 + c] * wts[j];
                tmp[((size_t)oy * w + x) * 3 + c] = t;
            }
    }
    /* horizontal pass: [nh][w] f32 -> [nh][nw] u8 */
    for (uint32_t ox = 0; ox < nw; ++ox) {
        uint32_t left;
        const uint32_t n = tri_window(w, nw, ox, wts, &left);
        for (uint32_t y = 0; y < nh; ++y)
            for (int c = 0; c < 3; ++c) {
                float t = 0.0f;
                for (uint32_t j = 0; j < n; ++j) t += tmp[((size_t)y * w + left + j) * 3 + c] * wts[j];
                if (t < 0.0f) t = 0.0f;
                if (t > 255.0f) t = 255.0f;
                dst[((size_t)y * nw + ox) * 3 + c] = (uint8_t)roundf(t);
            }
    }
    free(tmp);
    free(wts);
    return OR_OK;
}

/* RecPreprocess::process (rec.rs:60-105) written into a [3][H][stride] block: columns
 * [0, width) get the normalised pixels, [width, stride) are left untouched. */
static int process_into(const uint8_t *rgb, uint32_t w, uint32_t h, uint32_t target_h, uint32_t max_w, float *out,
                        uint32_t stride, uint32_t *out_w) {
    const uint32_t th = target_h > 1 ? target_h : 1;
    const uint32_t tw = oracle_rec_resized_width(w, h, target_h, max_w);
    uint8_t *img = (uint8_t *)malloc((size_t)tw * th * 3);
    if (!img) return OR_ERR_ARG;
    int rc = oracle_resize_triangle_rgb8(rgb, w, h, tw, th, img);
    if (rc) {
        free(img);
        return rc;
    }
    const float inv_127_5 = 1.0f / 127.5f;
    for (uint32_t y = 0; y < th; ++y)
        for (uint32_t x = 0; x < tw; ++x)
            for (int c = 0; c < 3; ++c)
                out[((size_t)c * th + y) * stride + x] = (float)img[((size_t)y * tw + x) * 3 + c] * inv_127_5 - 1.0f;
    free(img);
    *out_w = tw;
    return OR_OK;
}

/* One crop: out [3][H][width] with H = max(target_h, 1), width = oracle_rec_resized_width. */
int oracle_rec_preprocess(const uint8_t *rgb, uint32_t w, uint32_t h, uint32_t target_h, uint32_t max_w, float *out,
                          uint32_t *out_w) {
    const uint32_t tw = oracle_rec_resized_width(w, h, target_h, max_w);
    return process_into(rgb, w, h, target_h, max_w, out, tw, out_w);
}

typedef struct {
    const uint8_t *rgb;
    const int64_t *offsets;
    const uint32_t *widths, *heights;
    int64_t n_lines;
    uint32_t target_h, max_w, wmax;
    float *out;
    uint32_t *out_widths;
    int64_t next;
    pthread_mutex_t mu;
    int rc;
} batch_job;

static void *batch_worker(void *p) {
    batch_job *j = (batch_job *)p;
    const uint32_t th = j->target_h > 1 ? j->target_h : 1;
    const size_t line_floats = (size_t)3 * th * j->wmax;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        const int64_t l = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (l >= j->n_lines) break;
        float *dst = j->out + (size_t)l * line_floats;
        uint32_t tw = 0;
        const int rc = process_into(j->rgb + j->offsets[l], j->widths[l], j->heights[l], j->target_h, j->max_w, dst,
                                    j->wmax, &tw);
        if (rc) {
            pthread_mutex_lock(&j->mu);
            j->rc = rc;
            pthread_mutex_unlock(&j->mu);
            continue;
        }
        /* build_batch pads every row of every plane with white (+1.0) to Wmax */
        for (size_t r = 0; r < (size_t)3 * th; ++r)
            for (uint32_t x = tw; x < j->wmax; ++x) dst[r * j->wmax + x] = 1.0f;
        j->out_widths[l] = tw;
    }
    return NULL;
}

/* A batch of crops (crop l: RGB8 HWC at rgb + offsets[l], widths[l] x heights[l]) into
 * out [n_lines][3][H][wmax], wmax = the largest resized width, lines distributed over
 * `threads` workers (each runs its lines one at a time). */
int oracle_rec_preprocess_batch(const uint8_t *rgb, const int64_t *offsets, const uint32_t *widths,
                                const uint32_t *heights, int64_t n_lines, uint32_t target_h, uint32_t max_w,
                                float *out, uint32_t *out_widths, uint32_t *out_wmax, int threads) {
    uint32_t wmax = 0;
    for (int64_t l = 0; l < n_lines; ++l) {
        const uint32_t tw = oracle_rec_resized_width(widths[l], heights[l], target_h, max_w);
        if (tw > wmax) wmax = tw;
    }
    *out_wmax = wmax;
    if (n_lines <= 0) return OR_OK;
    batch_job j = {rgb, offsets, widths, heights, n_lines, target_h, max_w, wmax, out, out_widths, 0,
                   PTHREAD_MUTEX_INITIALIZER, OR_OK};
    if (threads < 1) threads = 1;
    if (threads == 1) {
        batch_worker(&j);
    } else {
        pthread_t *t = (pthread_t *)malloc((size_t)threads * sizeof(pthread_t));
        for (int i = 0; i < threads; ++i) pthread_create(&t[i], NULL, batch_worker, &j);
        for (int i = 0; i < threads; ++i) pthread_join(t[i], NULL);
        free(t);
    }
    return j.rc;
}
