// Launch parameters shared by the host dispatch (rechead_abi.cu) and the kernels
// (rechead_kernels.cu). Plain C types only.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace rh {

constexpr int kBlockM = 128;                  // timestep rows per work unit (one TMEM lane each)
constexpr int kBlockN = 128;                  // classes per weight tile / accumulator
constexpr int kPadK = 128;                    // K extent of a weight tile (K <= 128 supported)
constexpr int kTileBytes = kBlockN * kPadK * 2;  // one fp16 weight tile (the MMA's B operand): 32 KB
constexpr int kTile8Bytes = kBlockN * kPadK;  // one int8 weight tile as stored in HBM: 16 KB
constexpr int kCtabFloats = 2 * kBlockN;      // class table per tile: scale[128] then bias[128]
// Shared-memory weight ring (128 KB), by the form of the weight in HBM:
//  - fp16 image (rh_weight_pack): 4 stages of 32 KB, each filled by one bulk copy;
//  - int8 tiles (rh_weight_pack_compact): 3 fp16 stages filled by the expander warps from 2
//    int8 landing slots of 16 KB;
//  - FP32 hi/lo images (rh_weight_pack_f32): 2 stages of 64 KB.
constexpr int kStagesImage = 4;
constexpr int kStages8 = 3;
constexpr int kI8Slots = 2;
constexpr int kStagesDual = 2;

// Byte offset of class row r (0..127 within its tile) and K slot s (0..127) in an int8 tile:
// 16-byte chunks of 16 K slots, ordered [row group r/8][K chunk s/16][row r%8]. The expander
// warps read the tile as consecutive 16-byte chunks (conflict-free shared-memory loads) and
// each 8-lane phase writes 8 rows of one K chunk, whose swizzled fp16 positions are distinct
// (conflict-free stores).
__host__ __device__ constexpr uint32_t image8_offset(int r, int s) {
    return ((((uint32_t)(r >> 3) * 8u + (uint32_t)(s >> 4)) * 8u + (uint32_t)(r & 7)) << 4) + (uint32_t)(s & 15);
}
constexpr int kEpiGroups = 6;                 // epilogue warp groups (4 warps each)
constexpr int kHeadThreads = 32 * (8 + 4 * kEpiGroups);  // 32 warps, see head_kernel

// Device status word bits (status[0]); status[1] records which wait gave up.
constexpr int kDevTimeout = 1;
// Recognition preprocessing: a tap window or a staged column span exceeded the size the host
// planned for it (the access was skipped; never expected).
constexpr int kDevRecPlan = 2;
// Test-only: the weight producer never fills its stages, so every consumer's bounded wait
// runs out and the kernel must return kDevTimeout with the context intact.
constexpr int kDebugStallProducer = 1;
// Pairs of columns per 32-column quarter whose 2^x runs on the FMA pipe instead of MUFU.
// The epilogue is instruction-issue bound rather than MUFU bound, so the polynomial's extra
// instructions cost more than the MUFU time they save: 0 measured fastest on cfg2.
constexpr int kDefaultPolyPairs = 0;

struct HeadParams {
    const float* a;            // [m][k] timestep features (rows packed densely), or [b][k][t_len] (a_t > 0)
    long long a_t;             // 0: row-major rows; T > 0: a is the SVTR tail's [batch][k][T] (before
                               // Transpose.8), row r = (r / T, r % T) and element k sits T floats apart
    long long m;
    int k;
    int n;
    int n_chunks;              // ceil(n / 128)
    int hi_steps;              // MMA K-steps of the high fp16 part of A
    int lo_steps;              // MMA K-steps of the low fp16 part of A
    int merged_tail;           // 1: hi step hi_steps-1 also carries lo's last 8 K values
    const uint8_t* btiles;     // n_chunks tiles: fp16 image of 32 KB (shared-memory image order), or
                               // (expand) int8 of 16 KB (expansion order, q + 128), or (dual) fp16
                               // hi then lo image, 64 KB
    int dual;                  // FP32 weights: each tile holds fp16 hi and lo parts (A_hi.W_lo added)
    int expand;                // int8 tiles, expanded to fp16 in shared memory by warps 4-7
    const float* ctab;         // n_chunks * 256: per tile scale[128] then bias[128]; padded classes (0, -inf)
    int n_mblocks;             // ceil(m / 128)
    int whole_units;           // row blocks [0, whole_units) are units of the whole class range (full
                               // waves of the grid, no merge); the rest are split as below
    int n_splits;              // class-range splits per row block from whole_units on
    int chunks_per_split;
    int32_t* idx;              // fused, n_splits == 1: argmax class per row
    float* prob;               // fused, n_splits == 1: max softmax probability per row
    float4* partial;           // fused, n_splits > 1: [n_splits][m - 128 whole_units] (max, sum, idx bits,
                               // 0) of the split row blocks' rows, log2 units
    float* logits;             // logits variant: [m][n]
    int* status;               // [2]
    unsigned long long timeout_ns;
    int debug_flags;
    int poly_pairs;            // exp pairs per 64-class half computed on the FMA pipe (0,2,4,6,8)
};

struct PackParams {
    const float* w;            // [n][k] transposed head weight
    const float* bias;         // [n] or null
    int n;
    int k;
    int n_pad;                 // n_chunks * 128
    int merged_tail;
    int tail_step;             // index of the last hi K-step (ceil(k/16) - 1)
    int f32;                   // 1: FP32 weights (no int8): per-class power-of-two scale, fp16 hi + lo images
    int compact;               // quantised only: 1 = int8 tiles (16 KB), 0 = fp16 image tiles (32 KB)
    uint8_t* btiles;           // n_pad/128 tiles (f32: 64 KB, hi image then lo image)
    float* ctab;               // [n_pad / 128][256] scale then bias per tile
};

// Kernel launchers (rechead_kernels.cu).
cudaError_t launch_pack(const PackParams& p, cudaStream_t stream);
cudaError_t launch_head(const HeadParams& p, bool emit_logits, int grid, cudaStream_t stream);
cudaError_t launch_merge(const float4* partial, int n_splits, long long m, int32_t* idx, float* prob,
                         cudaStream_t stream);
// CTC greedy collapse of per-timestep (idx, prob) in device memory (ctc_kernels.cu). Line l is
// [line_offsets[l], line_offsets[l + 1]), or [line_offsets[l], line_ends[l]) when line_ends is given.
cudaError_t launch_ctc_collapse(const int32_t* idx, const float* prob, const int64_t* line_offsets, int64_t n_lines,
                                int32_t* tokens, int64_t* token_offsets, float* scores, cudaStream_t stream,
                                const int64_t* line_ends = nullptr);
size_t head_smem_bytes();
cudaError_t head_kernel_setup();

}  // namespace rh
