// CTC greedy collapse on the GPU: the loop of CtcDecoder::decode_batch
// (src/postprocess/ctc.rs:144-169) over per-timestep (argmax index, max probability) pairs
// that the fused head leaves in device memory, so that only the collapsed tokens and one
// score per line need to leave the GPU.
//
// For line l (timesteps [line_offsets[l], line_offsets[l+1])) timestep t emits idx[t] when
// idx[t] != 0 (blank) and idx[t] != idx[t-1] (the previous index starts at 0 for each line);
// the line's score is the f32 sum of the emitted probabilities in timestep order divided by
// their count (0 when none). Three launches:
//   ctc_count_kernel  one warp per line: number of emitted tokens -> token_offsets[l + 1]
//   ctc_scan_kernel   one block: token_offsets[0] = 0, inclusive scan of the counts
//   ctc_emit_kernel   one warp per line: compacts the emitted tokens to
//                     tokens[token_offsets[l]...] and computes the score. The score sum runs
//                     over the emitted probabilities in ascending t (every lane adds the
//                     same shuffled values in the same order), so it is bit-identical to the
//                     sequential host loop.
#include <cstdint>

#include "head_params.h"

namespace rh {

namespace {

constexpr int kCtcThreads = 256;  // 8 lines per block

// Line l owns timesteps [offs[l], offs[l + 1]), or [offs[l], ends[l]) when the lines have gaps
// between them (padded batches: ends given).
__device__ __forceinline__ void line_range(const int64_t* __restrict__ offs, const int64_t* __restrict__ ends,
                                           int64_t l, int64_t& b, int64_t& e) {
    b = offs[l];
    e = ends ? ends[l] : offs[l + 1];
    if (e < b) e = b;  // a decreasing pair is treated as an empty line (host entry points reject it)
}

__device__ __forceinline__ bool emits(const int32_t* __restrict__ idx, int64_t t, int64_t b, int64_t e,
                                      int32_t& c) {
    c = 0;
    if (t >= e) return false;
    c = idx[t];
    const int32_t prev = t > b ? idx[t - 1] : 0;
    return c != 0 && c != prev;
}

}  // namespace

__global__ void __launch_bounds__(kCtcThreads) ctc_count_kernel(const int32_t* __restrict__ idx,
                                                                 const int64_t* __restrict__ offs,
                                                                 const int64_t* __restrict__ ends, int64_t n_lines,
                                                                 int64_t* __restrict__ token_offsets) {
    const int64_t l = ((int64_t)blockIdx.x * kCtcThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (l >= n_lines) return;
    int64_t b, e;
    line_range(offs, ends, l, b, e);
    int64_t count = 0;
    for (int64_t t0 = b; t0 < e; t0 += 32) {
        int32_t c;
        const bool em = emits(idx, t0 + lane, b, e, c);
        count += __popc(__ballot_sync(0xffffffffu, em));
    }
    if (lane == 0) token_offsets[l + 1] = count;
}

__global__ void __launch_bounds__(1024) ctc_scan_kernel(int64_t* __restrict__ token_offsets, int64_t n_lines) {
    __shared__ int64_t warp_sums[32];
    __shared__ int64_t carry;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        token_offsets[0] = 0;
        carry = 0;
    }
    __syncthreads();
    for (int64_t base = 1; base <= n_lines; base += 1024) {
        const int64_t i = base + threadIdx.x;
        int64_t v = i <= n_lines ? token_offsets[i] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t u = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += u;
        }
        if (lane == 31) warp_sums[warp] = v;
        __syncthreads();
        if (warp == 0) {
            int64_t w = warp_sums[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t u = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += u;
            }
            warp_sums[lane] = w;  // inclusive over warps
        }
        __syncthreads();
        const int64_t add = carry + (warp > 0 ? warp_sums[warp - 1] : 0);
        if (i <= n_lines) token_offsets[i] = v + add;
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_sums[31];
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kCtcThreads) ctc_emit_kernel(const int32_t* __restrict__ idx,
                                                                const float* __restrict__ prob,
                                                                const int64_t* __restrict__ offs,
                                                                const int64_t* __restrict__ ends, int64_t n_lines,
                                                                const int64_t* __restrict__ token_offsets,
                                                                int32_t* __restrict__ tokens,
                                                                float* __restrict__ scores) {
    const int64_t l = ((int64_t)blockIdx.x * kCtcThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (l >= n_lines) return;
    int64_t b, e;
    line_range(offs, ends, l, b, e);
    int64_t pos = token_offsets[l];
    float sum = 0.0f;
    int64_t count = 0;
    const uint32_t below = (1u << lane) - 1u;
    for (int64_t t0 = b; t0 < e; t0 += 32) {
        int32_t c;
        const bool em = emits(idx, t0 + lane, b, e, c);
        const float p = em ? prob[t0 + lane] : 0.0f;
        const uint32_t mask = __ballot_sync(0xffffffffu, em);
        if (em) tokens[pos + __popc(mask & below)] = c;
        for (uint32_t m = mask; m; m &= m - 1u) sum += __shfl_sync(0xffffffffu, p, __ffs(m) - 1);
        pos += __popc(mask);
        count += __popc(mask);
    }
    if (lane == 0) scores[l] = count == 0 ? 0.0f : sum / (float)count;
}

cudaError_t launch_ctc_collapse(const int32_t* idx, const float* prob, const int64_t* line_offsets, int64_t n_lines,
                                int32_t* tokens, int64_t* token_offsets, float* scores, cudaStream_t stream,
                                const int64_t* line_ends) {
    const int64_t blocks = (n_lines * 32 + kCtcThreads - 1) / kCtcThreads;
    if (n_lines > 0)
        ctc_count_kernel<<<(unsigned)blocks, kCtcThreads, 0, stream>>>(idx, line_offsets, line_ends, n_lines,
                                                                       token_offsets);
    ctc_scan_kernel<<<1, 1024, 0, stream>>>(token_offsets, n_lines);
    if (n_lines > 0)
        ctc_emit_kernel<<<(unsigned)blocks, kCtcThreads, 0, stream>>>(idx, prob, line_offsets, line_ends, n_lines,
                                                                      token_offsets, tokens, scores);
    return cudaGetLastError();
}

}  // namespace rh
