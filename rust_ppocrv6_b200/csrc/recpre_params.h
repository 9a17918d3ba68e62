// Launch parameters of the batched recognition preprocessing, shared by the host dispatch
// (rechead_abi.cu) and the kernels (recpre_kernels.cu). Plain C types only.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace rh {

// Batched recognition preprocessing (recpre_kernels.cu): RecPreprocess::process of each crop
// (resize to out_h rows with the triangle filter, normalise to [-1, 1]) packed into one
// [n_lines][3][out_h][wmax] tensor whose columns past a line's width are +1.0 (white).
constexpr int kRecThreads = 256;   // threads per block
constexpr int kRecSpanMax = 12288; // most staged input columns (three f32 each: 144 KB of shared memory)
constexpr int kRecFastSlots = 4;   // weight slots per output column of a line with kx > 0 (one float4)
constexpr int kRecMetaMax = 4096;  // most column windows staged per block (80 KB)

struct RecLine {
    long long src;     // byte offset of the crop (RGB8, row-major HWC) in the pixel buffer
    int w, h;          // crop size in pixels; a zero means an empty crop (resized to black)
    int out_w;         // resized width
    int stride_x;      // weight slots per output column (>= its untrimmed tap count when kx == 0)
    int stride_y;      // weight slots per output row
    int chunk;         // output columns staged at once (1..out_w)
    int kx;            // 2..4: every column has at most kx non-zero taps (ceil(2 s), s <= 2), its weights
                       // zero-padded in a 16-byte aligned slot of kRecFastSlots = 4; 0: general columns
    long long coord;   // first (first tap, tap count) entry: out_w column entries, then out_h row entries
    long long wts;     // first weight (a multiple of 4): out_w * stride_x column weights, then out_h * stride_y
};

struct RecParams {
    const uint8_t* rgb;  // crops
    const RecLine* lines;
    long long n_lines;
    int out_h;           // rows per line (target height, at least 1)
    int wmax;            // columns per line in the output (the largest resized width)
    int span_cap;        // staged columns (shared memory: three f32 planes of span_cap)
    int meta_cap;        // column windows staged per block (0: none; lines with kx > 0, one chunk and
                         // out_w <= meta_cap stage theirs: float4 + f32 each)
    int2* coords;        // tap windows, trimmed to their non-zero weights
    float* wts;          // normalised tap weights
    float* out;          // [n_lines][3][out_h][wmax]
    float inv;           // 1 / 127.5 in f32
    int* status;         // [2]
};

// Tap windows and weights of every line (one launch), then the resize of lines [line0, line0 + n).
cudaError_t launch_rec_weights(const RecParams& p, cudaStream_t stream);
cudaError_t launch_rec_resize(const RecParams& p, long long line0, long long n, cudaStream_t stream);

}  // namespace rh
