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
// weights. Every operation is an IEEE f32 add, multiply or divide in the crate's order
// (__fadd_rn / __fmul_rn / __fdiv_rn: never contracted into an FMA), so the bytes are those of
// the crate and the floats those of process().
//
// Two launches:
//   rec_weights_kernel  one block per line: the tap window and normalised weights of each
//                       output column and row (computed once, reused by every row / column).
//   rec_resize_kernel   one block per (line, output row y): for chunks of up to 256 output
//                       columns, the vertical pass of the chunk's input column span into
//                       shared memory (3 channel planes), then the horizontal pass, one output
//                       column per thread, writing the three normalised planes (coalesced),
//                       then the white padding up to wmax. HBM-bound: every crop byte is read
//                       from DRAM about once (the rows a block shares with its neighbours come
//                       from L2) and every output float is written once.
#include <cstdint>

#include "head_params.h"

namespace rh {

namespace {

__device__ __forceinline__ void flag(int* status) { atomicOr(status, kDevRecPlan); }

// Tap window of output coordinate o (first tap, count) and its normalised weights in w[0..count).
__device__ int2 tri_window(int n_in, int n_out, int o, int stride, float* __restrict__ w, int* status) {
    const float ratio = __fdiv_rn((float)n_in, (float)n_out);
    const float s = ratio < 1.0f ? 1.0f : ratio;
    const float centre = __fmul_rn(__fadd_rn((float)o, 0.5f), ratio);
    long long lo = (long long)floorf(__fsub_rn(centre, s));
    lo = lo < 0 ? 0 : (lo > n_in - 1 ? n_in - 1 : lo);
    long long hi = (long long)ceilf(__fadd_rn(centre, s));
    hi = hi < lo + 1 ? lo + 1 : hi;
    hi = hi > n_in ? n_in : hi;
    int cnt = (int)(hi - lo);
    if (cnt > stride) {  // the host sized the slots from 2s + 3; never expected
        flag(status);
        cnt = stride;
    }
    const float c0 = __fsub_rn(centre, 0.5f);
    float sum = 0.0f;
    for (int j = 0; j < cnt; ++j) {
        const float x = fabsf(__fdiv_rn(__fsub_rn((float)(lo + j), c0), s));
        const float wj = x < 1.0f ? __fsub_rn(1.0f, x) : 0.0f;
        w[j] = wj;
        sum = __fadd_rn(sum, wj);
    }
    for (int j = 0; j < cnt; ++j) w[j] = __fdiv_rn(w[j], sum);
    return make_int2((int)lo, cnt);
}

// Clamp to [0, 255], round half away from zero (the u8 of the resized image), normalise.
__device__ __forceinline__ float to_unit(float t, float inv) {
    t = t < 0.0f ? 0.0f : (t > 255.0f ? 255.0f : t);
    return __fsub_rn(__fmul_rn(roundf(t), inv), 1.0f);
}

}  // namespace

__global__ void __launch_bounds__(kRecThreads) rec_weights_kernel(const RecParams p) {
    const RecLine L = p.lines[blockIdx.x];
    if (L.w <= 0 || L.h <= 0) return;  // empty crop: black, no taps
    const int n = L.out_w + p.out_h;
    for (int j = threadIdx.x; j < n; j += kRecThreads) {
        if (j < L.out_w) {
            p.coords[L.coord + j] =
                tri_window(L.w, L.out_w, j, L.stride_x, p.wts + L.wts + (long long)j * L.stride_x, p.status);
        } else {
            const int y = j - L.out_w;
            p.coords[L.coord + j] = tri_window(L.h, p.out_h, y, L.stride_y,
                                               p.wts + L.wts + (long long)L.out_w * L.stride_x +
                                                   (long long)y * L.stride_y,
                                               p.status);
        }
    }
}

__global__ void __launch_bounds__(kRecThreads) rec_resize_kernel(const RecParams p, long long line0) {
    extern __shared__ float vs[];  // [3][span_cap]: vertical-pass values of the chunk's input columns
    const long long li = line0 + blockIdx.x / p.out_h;
    const int y = (int)(blockIdx.x % p.out_h);
    const RecLine L = p.lines[li];
    const size_t plane = (size_t)p.out_h * (size_t)p.wmax;
    float* r0 = p.out + (size_t)li * 3 * plane + (size_t)y * (size_t)p.wmax;
    float* r1 = r0 + plane;
    float* r2 = r1 + plane;
    for (int x = L.out_w + threadIdx.x; x < p.wmax; x += kRecThreads) {  // white padding (batch_poc.rs:18-19)
        r0[x] = 1.0f;
        r1[x] = 1.0f;
        r2[x] = 1.0f;
    }
    if (L.w <= 0 || L.h <= 0) {  // an empty crop resizes to black
        for (int x = threadIdx.x; x < L.out_w; x += kRecThreads) {
            r0[x] = -1.0f;
            r1[x] = -1.0f;
            r2[x] = -1.0f;
        }
        return;
    }
    const int2 cy = p.coords[L.coord + L.out_w + y];
    const float* __restrict__ wy = p.wts + L.wts + (long long)L.out_w * L.stride_x + (long long)y * L.stride_y;
    const size_t pitch = (size_t)L.w * 3;
    const uint8_t* __restrict__ top = p.rgb + L.src + (size_t)cy.x * pitch;
    const int cap = p.span_cap;
    for (int x0 = 0; x0 < L.out_w; x0 += L.chunk) {
        const int x1 = min(x0 + L.chunk, L.out_w);
        const int2 a = p.coords[L.coord + x0], b = p.coords[L.coord + x1 - 1];
        const int left0 = a.x, span = b.x + b.y - a.x;
        if (span <= 0 || span > cap) {  // same values in every thread: the whole block leaves
            if (threadIdx.x == 0) flag(p.status);
            return;
        }
        // vertical pass over input columns [left0, left0 + span): taps in order, f32
        for (int c = threadIdx.x; c < span; c += kRecThreads) {
            const uint8_t* __restrict__ px = top + (size_t)(left0 + c) * 3;
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f;
            for (int i = 0; i < cy.y; ++i) {
                const float wv = __ldg(wy + i);
                a0 = __fadd_rn(a0, __fmul_rn((float)__ldg(px), wv));
                a1 = __fadd_rn(a1, __fmul_rn((float)__ldg(px + 1), wv));
                a2 = __fadd_rn(a2, __fmul_rn((float)__ldg(px + 2), wv));
                px += pitch;
            }
            vs[c] = a0;
            vs[cap + c] = a1;
            vs[2 * cap + c] = a2;
        }
        __syncthreads();
        // horizontal pass: one output column per thread
        const int x = x0 + (int)threadIdx.x;
        if (x < x1) {
            const int2 cx = p.coords[L.coord + x];
            const float* __restrict__ wx = p.wts + L.wts + (long long)x * L.stride_x;
            const int base = cx.x - left0;
            if (base >= 0 && base + cx.y <= span) {
                float t0 = 0.0f, t1 = 0.0f, t2 = 0.0f;
                for (int j = 0; j < cx.y; ++j) {
                    const float wv = __ldg(wx + j);
                    t0 = __fadd_rn(t0, __fmul_rn(vs[base + j], wv));
                    t1 = __fadd_rn(t1, __fmul_rn(vs[cap + base + j], wv));
                    t2 = __fadd_rn(t2, __fmul_rn(vs[2 * cap + base + j], wv));
                }
                r0[x] = to_unit(t0, p.inv);
                r1[x] = to_unit(t1, p.inv);
                r2[x] = to_unit(t2, p.inv);
            } else {
                flag(p.status);
            }
        }
        __syncthreads();
    }
}

cudaError_t launch_rec_weights(const RecParams& p, cudaStream_t stream) {
    if (p.n_lines <= 0) return cudaSuccess;
    rec_weights_kernel<<<(unsigned)p.n_lines, kRecThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_rec_resize(const RecParams& p, long long line0, long long n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const size_t smem = (size_t)3 * (size_t)p.span_cap * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(rec_resize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    rec_resize_kernel<<<(unsigned)(n * p.out_h), kRecThreads, smem, stream>>>(p, line0);
    return cudaGetLastError();
}

}  // namespace rh
