// Batched recognition preprocessing on the GPU: RecPreprocess::process
// (src/preprocess/rec.rs:60-105) of every crop of a batch, packed the way the reference's
// batching proof of concept does it (tools/profiling/batch_poc.rs:14-32): one
// [n_lines][3][H][wmax] f32 tensor, channel planes, columns past a line's width = +1.0.
//
// The resize is the `image` crate's resize_exact(w, H, FilterType::Triangle) (image 0.25,
// separable): a vertical pass to f32, then a horizontal pass that clamps to [0, 255] and
// rounds half away from zero, then v / 127.5 - 1 (as v * (1/127.5) - 1). Output coordinate o
// of an n_in -> n_out axis has ratio = n_in / n_out, s = max(ratio, 1), centre (o + 1/2) *
// ratio, taps [floor(centre - s), ceil(centre + s)) clipped to the image (at least one), tap i
// weighing max(0, 1 - |(i - (centre - 1/2)) / s|) divided by the f32 sum of the window's
// weights; every sum runs over the taps in order. Every operation here is an IEEE f32 add,
// multiply or divide in that order (__fadd_rn / __fmul_rn / __fdiv_rn: never contracted into
// an FMA), so the bytes are those of the crate and the floats those of process().
//
// Exact shortcuts. Each product is >= +0 (bytes and weights are >= 0), so a running sum never
// changes when a zero-weight tap is added: the weight tables drop the zero taps at the ends of
// each window, padded slots carry weight 0, and the first tap's sum 0 + p*w is written p*w.
// A window's non-zero taps are the integers i with |i - c'| < s, at most ceil(2 s) of them
// (f32 rounding is monotone, so it never admits a tap the real-valued test rejects).
//
// Two launches:
//   rec_weights_kernel  one thread per (line, output column or row): the trimmed tap window and
//                       normalised weights (computed once, reused by every row / column).
//   rec_resize_kernel   one block per (line, 8 output rows). The white padding first; then per
//                       row and chunk of output columns (the whole line unless its input span is
//                       very wide): the vertical pass of the chunk's input columns into shared
//                       memory (three f32 planes, taps unrolled for the row's tap count, weights
//                       in registers), then the horizontal pass (unrolled to the line's bound kx),
//                       writing the three normalised planes (coalesced). A one-chunk line with
//                       kx > 0 stages its column windows in shared memory once for all 8 rows
//                       (they do not depend on the row): one 16-byte record per column. Each crop
//                       byte is read from DRAM about once (rows shared with neighbouring blocks
//                       come from L2) and each output float is written once; the kernel is bound
//                       by the L1 / shared-memory data pipe (the byte loads, the stage and its
//                       reads), not by HBM.
#include <cstdint>

#include "head_params.h"
#include "recpre_params.h"

namespace rh {

namespace {

constexpr int kRecRows = 8;  // output rows per block (consecutive: they share input rows and column tables)

__device__ __forceinline__ void flag(int* status) { atomicOr(status, kDevRecPlan); }

// Tap window of output coordinate o, trimmed to its non-zero weights: returns (first tap,
// count) and leaves the normalised weights in w[0..count), zeros in w[count..pad).
// Windows of up to 8 taps (every axis that shrinks by at most 3x) are computed in registers
// and written once; wider ones go through w itself. The slots hold at least the trimmed window
// (stride >= count); the loop for wider windows needs the untrimmed one (stride >= hi - lo).
// A slot of exactly 4 (pad == stride == 4) is written whole by one 16-byte store, so the L2
// never has to merge a partly written sector with DRAM. Divisions whose result is known
// exactly are not carried out: those of the slots past the window, d / s when s == 1 and
// w / sum when sum == 1.
__device__ __forceinline__ int2 tri_window(int n_in, int n_out, int o, int stride, int pad, float* __restrict__ w, int* status) {
    const float ratio = __fdiv_rn((float)n_in, (float)n_out);
    const float s = ratio < 1.0f ? 1.0f : ratio;
    const float centre = __fmul_rn(__fadd_rn((float)o, 0.5f), ratio);
    long long lo = (long long)floorf(__fsub_rn(centre, s));
    lo = lo < 0 ? 0 : (lo > n_in - 1 ? n_in - 1 : lo);
    long long hi = (long long)ceilf(__fadd_rn(centre, s));
    hi = hi < lo + 1 ? lo + 1 : hi;
    hi = hi > n_in ? n_in : hi;
    int cnt = (int)(hi - lo);
    if (cnt > 8 && cnt > stride) {  // the host sized the slots from 2s + 3; never expected
        flag(status);
        cnt = stride;
    }
    const float c0 = __fsub_rn(centre, 0.5f);
    float sum = 0.0f;
    if (cnt <= 8) {
        float r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float rj = 0.0f;
            if (j < cnt) {  // d / s is d exactly when s == 1 (every axis that grows)
                const float d = __fsub_rn((float)(lo + j), c0);
                const float x = fabsf(s == 1.0f ? d : __fdiv_rn(d, s));
                rj = x < 1.0f ? __fsub_rn(1.0f, x) : 0.0f;
            }
            r[j] = rj;
            sum = __fadd_rn(sum, rj);  // taps past cnt add +0: the sum is unchanged
        }
        int j0 = cnt, j1 = -1;  // first and last non-zero tap
#pragma unroll
        for (int j = 7; j >= 0; --j) j0 = r[j] != 0.0f ? j : j0;
#pragma unroll
        for (int j = 0; j < 8; ++j) j1 = r[j] != 0.0f ? j : j1;
        if (j1 < j0) j0 = j1 = 0;  // no non-zero tap (a zero sum; never expected): keep one
        int n = j1 - j0 + 1;
        if (n > stride) {  // a kx > 0 slot holds ceil(2 s) >= n taps; never expected
            flag(status);
            n = stride;
        }
        const int m = max(n, min(pad, stride));  // slots to write
        // q = r shifted down by j0, in three conditional steps of 1, 2 and 4 (every index is a
        // constant, so r and q stay in registers)
        float q[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) q[k] = r[k];
#pragma unroll
        for (int st = 1; st < 8; st <<= 1) {
            if (j0 & st) {
#pragma unroll
                for (int k = 0; k < 8; ++k) q[k] = k + st < 8 ? q[k + st] : 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (k >= n) q[k] = 0.0f;
            else if (sum != 1.0f) q[k] = __fdiv_rn(q[k], sum);  // v / 1 is v exactly
        }
        if (pad == 4 && stride == 4) {
            *reinterpret_cast<float4*>(w) = make_float4(q[0], q[1], q[2], q[3]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (k < m) w[k] = q[k];
        }
        return make_int2((int)lo + j0, n);
    }
    for (int j = 0; j < cnt; ++j) {
        const float x = fabsf(__fdiv_rn(__fsub_rn((float)(lo + j), c0), s));
        const float wj = x < 1.0f ? __fsub_rn(1.0f, x) : 0.0f;
        w[j] = wj;
        sum = __fadd_rn(sum, wj);
    }
    int j0 = 0, j1 = cnt - 1;
    for (int j = 0; j < cnt; ++j) w[j] = __fdiv_rn(w[j], sum);
    while (j0 < j1 && w[j0] == 0.0f) ++j0;
    while (j1 > j0 && w[j1] == 0.0f) --j1;
    const int n = j1 - j0 + 1;
    if (j0 > 0)
        for (int j = 0; j < n; ++j) w[j] = w[j + j0];
    for (int j = n; j < pad && j < stride; ++j) w[j] = 0.0f;
    return make_int2((int)lo + j0, n);
}

// Clamp to 255 (the sum is never negative), round half away from zero (the u8 of the resized
// image), normalise. The rounding is one fused multiply-add rounding toward -inf:
// 24929 * 336.5 = 2^23 + 1/2 exactly, so for 0 <= t <= 255 the exact value 2^23 + 1/2 + t lies
// in [2^23, 2^24), where the floats are the integers, and rounding it down gives
// 2^23 + floor(t + 1/2) = 2^23 + round(t) (a tie goes up, i.e. away from zero, for t >= 0).
// Removing 2^23 is exact.
__device__ __forceinline__ float to_unit(float t, float inv) {
    t = fminf(t, 255.0f);
    const float n = __fadd_rn(__fmaf_rd(24929.0f, 336.5f, t), -8388608.0f);
    return __fsub_rn(__fmul_rn(n, inv), 1.0f);
}

// The vertical-pass stage in shared memory: one f32 plane per channel, span_cap columns each
// (three 4-byte reads per tap: a warp's taps spread over about 32 s consecutive columns, so
// each read costs about ceil(s) bank passes, and no lane of padding is moved).
struct Stage {
    float* r;
    float* g;
    float* b;
};

// (pr, pg, pb) * w added to a channel accumulator (the first tap sets it).
__device__ __forceinline__ void tap(float4& a, float pr, float pg, float pb, float w, bool first) {
    if (first) {
        a.x = __fmul_rn(pr, w);
        a.y = __fmul_rn(pg, w);
        a.z = __fmul_rn(pb, w);
    } else {
        a.x = __fadd_rn(a.x, __fmul_rn(pr, w));
        a.y = __fadd_rn(a.y, __fmul_rn(pg, w));
        a.z = __fadd_rn(a.z, __fmul_rn(pb, w));
    }
}

__device__ __forceinline__ void tap(float4& a, float4 p, float w, bool first) { tap(a, p.x, p.y, p.z, w, first); }

// Staged column c as a tap.
__device__ __forceinline__ void tap(float4& a, const Stage& st, int c, float w, bool first) {
    tap(a, st.r[c], st.g[c], st.b[c], w, first);
}

__device__ __forceinline__ void put(const Stage& st, int c, const float4& a) {
    st.r[c] = a.x;
    st.g[c] = a.y;
    st.b[c] = a.z;
}

__device__ __forceinline__ float4 px3(const uint8_t* __restrict__ p) {
    return make_float4((float)__ldg(p), (float)__ldg(p + 1), (float)__ldg(p + 2), 0.0f);
}

// Vertical pass of input columns [left0, left0 + span) for a row with NY taps starting at
// `top` (NY == 0: any count, loop). Each thread takes U columns per step, loading all their
// bytes before the arithmetic so that the loads overlap.
template <int NY, int U>
__device__ __forceinline__ void vpass(const Stage st, const uint8_t* __restrict__ top, size_t pitch, int left0,
                                      int span, const float* __restrict__ wy, int ny) {
    if constexpr (NY == 0) {
        for (int c = threadIdx.x; c < span; c += kRecThreads) {
            const uint8_t* __restrict__ q = top + (size_t)(left0 + c) * 3;
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int j = 0; j < ny; ++j) tap(a, px3(q + j * pitch), __ldg(wy + j), j == 0);
            put(st, c, a);
        }
    } else {
        float w[NY];
#pragma unroll
        for (int j = 0; j < NY; ++j) w[j] = __ldg(wy + j);
        for (int c0 = threadIdx.x; c0 < span; c0 += U * kRecThreads) {
            float4 v[U][NY];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = min(c0 + u * kRecThreads, span - 1);  // a clamped column is loaded, not stored
                const uint8_t* __restrict__ q = top + (size_t)(left0 + c) * 3;
#pragma unroll
                for (int j = 0; j < NY; ++j) v[u][j] = px3(q + j * pitch);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int j = 0; j < NY; ++j) tap(a, v[u][j], w[j], j == 0);
                if (c0 + u * kRecThreads < span) put(st, c0 + u * kRecThreads, a);
            }
        }
    }
}

// Horizontal pass of output columns [x0, x1): at most KX taps per column (KX == 0: any
// count). Each thread takes U columns per step, loading their windows first.
template <int KX, int U>
__device__ __forceinline__ void hpass(const RecParams& p, const RecLine& L, const Stage st, int left0, int span,
                                      int x0, int x1, float* r0, float* r1, float* r2) {
    const int last = span - 1;
    for (int xb = x0 + (int)threadIdx.x; xb < x1; xb += U * kRecThreads) {
        int2 cx[U];
        float4 w4[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int x = min(xb + u * kRecThreads, x1 - 1);
            cx[u] = p.coords[L.coord + x];
            if (KX > 0) w4[u] = __ldg(reinterpret_cast<const float4*>(p.wts + L.wts + (long long)x * L.stride_x));
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int x = xb + u * kRecThreads;
            if (x >= x1) break;
            const int base = cx[u].x - left0;
            if (base < 0 || base + cx[u].y > span) {
                flag(p.status);
                continue;
            }
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            if (KX > 0 && cx[u].y <= KX) {
                const float wv[4] = {w4[u].x, w4[u].y, w4[u].z, w4[u].w};
#pragma unroll
                for (int j = 0; j < (KX > 0 ? KX : 1); ++j) tap(a, st, min(base + j, last), wv[j], j == 0);
            } else {
                const float* __restrict__ wx = p.wts + L.wts + (long long)x * L.stride_x;
                for (int j = 0; j < cx[u].y; ++j) tap(a, st, base + j, __ldg(wx + j), j == 0);
            }
            r0[x] = to_unit(a.x, p.inv);
            r1[x] = to_unit(a.y, p.inv);
            r2[x] = to_unit(a.z, p.inv);
        }
    }
}

// Horizontal pass of a whole line (one chunk) whose column windows were staged once per block:
// mrec[x] = (first tap relative to the staged span, as int bits; weights 0..2), mw3[x] = weight 3,
// zero-padded (a window that failed its check has weight 0 and raised the status flag): one
// 16-byte read per column for KX <= 3. The stage holds 4 zero columns past the span, so a padded
// tap reads a finite value and adds exactly 0. Branch-free: the last step's spare lanes
// recompute column out_w - 1 and do not store.
template <int KX, int U>
__device__ __forceinline__ void hpass_staged(const Stage st, const float4* __restrict__ mrec,
                                             const float* __restrict__ mw3, int out_w, float inv, float* r0,
                                             float* r1, float* r2) {
    for (int xb = (int)threadIdx.x; xb < out_w; xb += U * kRecThreads) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int x = xb + u * kRecThreads;
            const int xc = min(x, out_w - 1);
            const float4 m = mrec[xc];
            const int base = __float_as_int(m.x);
            const float wv[4] = {m.y, m.z, m.w, KX > 3 ? mw3[xc] : 0.0f};
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < KX; ++j) tap(a, st, base + j, wv[j], j == 0);
            if (x < out_w) {
                r0[x] = to_unit(a.x, inv);
                r1[x] = to_unit(a.y, inv);
                r2[x] = to_unit(a.z, inv);
            }
        }
    }
}

}  // namespace

__global__ void __launch_bounds__(kRecThreads) rec_weights_kernel(const RecParams p) {
    const RecLine L = p.lines[blockIdx.x];
    if (L.w <= 0 || L.h <= 0) return;  // empty crop: black, no taps
    const int j = blockIdx.y * kRecThreads + threadIdx.x;  // output column j, or row j - out_w
    if (j < L.out_w) {
        p.coords[L.coord + j] = tri_window(L.w, L.out_w, j, L.stride_x, L.kx > 0 ? 4 : 0,
                                           p.wts + L.wts + (long long)j * L.stride_x, p.status);
    } else if (j < L.out_w + p.out_h) {
        const int y = j - L.out_w;
        p.coords[L.coord + j] = tri_window(L.h, p.out_h, y, L.stride_y, 0,
                                           p.wts + L.wts + (long long)L.out_w * L.stride_x + (long long)y * L.stride_y,
                                           p.status);
    }
}

__global__ void __launch_bounds__(kRecThreads, 6) rec_resize_kernel(const RecParams p, long long line0) {
    // three f32 planes [span_cap]: the vertical-pass values (r, g, b) of the chunk's columns; then,
    // 16-byte aligned, for the staged column windows float4 [meta_cap] records and f32 [meta_cap]
    // fourth weights
    extern __shared__ float4 smem[];
    float* const planes = reinterpret_cast<float*>(smem);
    const Stage st{planes, planes + p.span_cap, planes + 2 * p.span_cap};
    const int groups = (p.out_h + kRecRows - 1) / kRecRows;
    const long long li = line0 + blockIdx.x / groups;
    const int y0 = (int)(blockIdx.x % groups) * kRecRows, y1 = min(y0 + kRecRows, p.out_h);
    const RecLine L = p.lines[li];
    const size_t plane = (size_t)p.out_h * (size_t)p.wmax;
    float* const line_out = p.out + (size_t)li * 3 * plane;
    const bool empty = L.w <= 0 || L.h <= 0;
    for (int y = y0; y < y1; ++y) {  // white padding (batch_poc.rs:18-19); an empty crop is black
        float* r0 = line_out + (size_t)y * (size_t)p.wmax;
        for (int x = (empty ? 0 : L.out_w) + threadIdx.x; x < p.wmax; x += kRecThreads) {
            const float v = x < L.out_w ? -1.0f : 1.0f;
            r0[x] = v;
            r0[x + plane] = v;
            r0[x + 2 * plane] = v;
        }
    }
    if (empty) return;
    const size_t pitch = (size_t)L.w * 3;
    if (L.kx > 0 && L.chunk == L.out_w && L.out_w <= p.meta_cap) {
        // One chunk per row and at most kx taps per column: the column windows do not depend on
        // the row, so they are staged once for the block's rows.
        float4* mrec = smem + (3 * p.span_cap + 3) / 4;
        float* mw3 = reinterpret_cast<float*>(mrec + p.meta_cap);
        const int2 a = p.coords[L.coord], b = p.coords[L.coord + L.out_w - 1];
        const int left0 = a.x, span = b.x + b.y - a.x;
        if (span <= 0 || span + 4 > p.span_cap) {  // same values in every thread: the whole block leaves
            if (threadIdx.x == 0) flag(p.status);
            return;
        }
        for (int x = threadIdx.x; x < L.out_w; x += kRecThreads) {
            const int2 cx = p.coords[L.coord + x];
            const int base = cx.x - left0;
            const bool ok = base >= 0 && base + cx.y <= span && cx.y <= L.kx;
            if (!ok) flag(p.status);
            const float4 w = ok ? __ldg(reinterpret_cast<const float4*>(p.wts + L.wts + (long long)x * L.stride_x))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
            mrec[x] = make_float4(__int_as_float(ok ? base : 0), w.x, w.y, w.z);
            mw3[x] = w.w;
        }
        if (threadIdx.x < 4) put(st, span + threadIdx.x, make_float4(0.f, 0.f, 0.f, 0.f));  // tap padding
        for (int y = y0; y < y1; ++y) {
            const int2 cy = p.coords[L.coord + L.out_w + y];
            const float* __restrict__ wy = p.wts + L.wts + (long long)L.out_w * L.stride_x + (long long)y * L.stride_y;
            const uint8_t* __restrict__ top = p.rgb + L.src + (size_t)cy.x * pitch;
            float* r0 = line_out + (size_t)y * (size_t)p.wmax;
            if (y > y0) __syncthreads();  // the previous horizontal pass is done with the stage
            switch (cy.y) {
                case 1: vpass<1, 2>(st, top, pitch, left0, span, wy, 1); break;
                case 2: vpass<2, 2>(st, top, pitch, left0, span, wy, 2); break;
                case 3: vpass<3, 2>(st, top, pitch, left0, span, wy, 3); break;
                case 4: vpass<4, 1>(st, top, pitch, left0, span, wy, 4); break;
                default: vpass<0, 1>(st, top, pitch, left0, span, wy, cy.y); break;
            }
            __syncthreads();  // also publishes mrec / mw3 before the first row's horizontal pass
            switch (L.kx) {
                case 2: hpass_staged<2, 1>(st, mrec, mw3, L.out_w, p.inv, r0, r0 + plane, r0 + 2 * plane); break;
                case 3: hpass_staged<3, 1>(st, mrec, mw3, L.out_w, p.inv, r0, r0 + plane, r0 + 2 * plane); break;
                default: hpass_staged<4, 1>(st, mrec, mw3, L.out_w, p.inv, r0, r0 + plane, r0 + 2 * plane); break;
            }
        }
        return;
    }
    for (int y = y0; y < y1; ++y) {
        const int2 cy = p.coords[L.coord + L.out_w + y];
        const float* __restrict__ wy = p.wts + L.wts + (long long)L.out_w * L.stride_x + (long long)y * L.stride_y;
        const uint8_t* __restrict__ top = p.rgb + L.src + (size_t)cy.x * pitch;
        float* r0 = line_out + (size_t)y * (size_t)p.wmax;
        float* r1 = r0 + plane;
        float* r2 = r1 + plane;
        for (int x0 = 0; x0 < L.out_w; x0 += L.chunk) {
            const int x1 = min(x0 + L.chunk, L.out_w);
            const int2 a = p.coords[L.coord + x0], b = p.coords[L.coord + x1 - 1];
            const int left0 = a.x, span = b.x + b.y - a.x;
            if (span <= 0 || span > p.span_cap) {  // same values in every thread: the whole block leaves
                if (threadIdx.x == 0) flag(p.status);
                return;
            }
            if (y > y0 || x0 > 0) __syncthreads();  // the previous horizontal pass is done with the stage
            switch (cy.y) {
                case 1: vpass<1, 2>(st, top, pitch, left0, span, wy, 1); break;
                case 2: vpass<2, 2>(st, top, pitch, left0, span, wy, 2); break;
                case 3: vpass<3, 2>(st, top, pitch, left0, span, wy, 3); break;
                case 4: vpass<4, 1>(st, top, pitch, left0, span, wy, 4); break;
                default: vpass<0, 1>(st, top, pitch, left0, span, wy, cy.y); break;
            }
            __syncthreads();
            switch (L.kx) {
                case 2: hpass<2, 1>(p, L, st, left0, span, x0, x1, r0, r1, r2); break;
                case 3: hpass<3, 1>(p, L, st, left0, span, x0, x1, r0, r1, r2); break;
                case 4: hpass<4, 1>(p, L, st, left0, span, x0, x1, r0, r1, r2); break;
                default: hpass<0, 1>(p, L, st, left0, span, x0, x1, r0, r1, r2); break;
            }
        }
    }
}

cudaError_t launch_rec_weights(const RecParams& p, cudaStream_t stream) {
    if (p.n_lines <= 0) return cudaSuccess;
    const dim3 grid((unsigned)p.n_lines, (unsigned)((p.wmax + p.out_h + kRecThreads - 1) / kRecThreads));
    rec_weights_kernel<<<grid, kRecThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_rec_resize(const RecParams& p, long long line0, long long n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const size_t smem = (size_t)((3 * p.span_cap + 3) / 4) * sizeof(float4) +
                        (size_t)p.meta_cap * (sizeof(float4) + sizeof(float));
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(rec_resize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const long long groups = (p.out_h + kRecRows - 1) / kRecRows;
    rec_resize_kernel<<<(unsigned)(n * groups), kRecThreads, smem, stream>>>(p, line0);
    return cudaGetLastError();
}

}  // namespace rh
