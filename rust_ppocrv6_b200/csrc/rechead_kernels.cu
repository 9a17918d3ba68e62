// sm_100a kernels of the quantised recognition head (PP-OCRv6 small rec, graph nodes
// MatMul.12 + Add.204 -> Softmax.2 -> CTC greedy argmax):
//
//  pack_kernel   QuantizedWeight::from_f32_transposed (src/ops/matmul.rs:1173-1202) on the
//                GPU: per-class symmetric int8 + f32 scale, bit-exact; also writes the
//                tensor-core image of the weight (fp16 tiles in shared-memory order) and the
//                per-class epilogue tables.
//  pack_f32_kernel  the FP32 head's weight (matmul_transposed_b, src/ops/matmul.rs:514-897):
//                per-class power-of-two scale, fp16 hi and lo images, epilogue tables.
//  head_kernel   persistent, warp-specialised W8A32 (or FP32) projection. A (f32 features) is split
//                into two fp16 parts in TMEM, weight tiles stream in through TMA bulk copies,
//                tcgen05.mma accumulates in TMEM, and the epilogue applies scale + bias and
//                either
//                  - FUSED: keeps an online (max, sum exp, first argmax) per row, so only
//                    idx/prob leave the chip (matmul_quantized_b + softmax_inplace +
//                    find_argmax, src/ops/matmul.rs:1204, src/ops/softmax.rs:199,
//                    src/postprocess/ctc.rs:178), or
//                  - LOGITS: writes the full [m][n] logits (the literal MatMul.12 output).
//  merge_kernel  combines per-split partial (max, sum, idx) triples when the class range of
//                a row block was split across CTAs.
#include <cuda_fp16.h>
#include <math_constants.h>

#include "head_params.h"
#include "sm100_ptx.cuh"

namespace rh {

namespace {

constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- shared memory map
// (offsets from the 1024-byte aligned base)
// Weight ring (128 KB): fp16 image weights kStagesImage stages of 32 KB (the MMA's B operand);
// int8 tiles kStages8 fp16 stages at [0, 96 KB), then kI8Slots int8 landing slots of 16 KB;
// FP32 weights kStagesDual stages of 64 KB (hi image, then lo image).
constexpr uint32_t kOffB = 0;
constexpr uint32_t kOffI8 = kStages8 * kTileBytes;
constexpr uint32_t kWeightRegion = kOffI8 + kI8Slots * kTile8Bytes;
static_assert(kWeightRegion >= (uint32_t)kStagesDual * 2u * kTileBytes &&
                  kWeightRegion >= (uint32_t)kStagesImage * kTileBytes,
              "every form's stages fit the weight ring");
constexpr uint32_t kOffBars = kWeightRegion;                    // mbarriers (48 x 8 B)
constexpr uint32_t kOffMisc = kOffBars + 48 * 8;                // [0] TMEM base, [1] abort flag
constexpr uint32_t kOffRho = kOffMisc + 32;                     // [4][128] f32 row de-scale
constexpr uint32_t kOffQFlag = kOffRho + 4 * 128 * 4;           // [4][4] u32 "quadrant needs de-scale"
constexpr uint32_t kOffMerge = kOffQFlag + 16 * 4;              // [2][kEpiGroups-1][128] float4
constexpr uint32_t kOffCtab = kOffMerge + 2 * (kEpiGroups - 1) * 128 * 16;  // [4 slots][256] f32 class table
constexpr uint32_t kCtabSlots = 4;
constexpr uint32_t kCtabBytes = kCtabFloats * 4;
constexpr uint32_t kOffRowMax = kOffCtab + kCtabSlots * kCtabBytes;  // [128] u64 (unit tag, ordered max)
constexpr uint32_t kOffAStage = kOffRowMax + 128 * 8;           // [128][k] f32 feature rows of a unit
constexpr uint32_t kAStageBytes = kBlockM * kPadK * 4;
constexpr uint32_t kSmemUsed = kOffAStage + kAStageBytes;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;               // + alignment slack
static_assert(kOffCtab % 16 == 0 && kOffAStage % 16 == 0 && kOffI8 % 1024 == 0, "bulk-copy destination alignment");
static_assert(kSmemUsed + 1024 <= 227 * 1024, "shared memory per CTA");

// mbarrier indices
constexpr int kMaxStages = kStagesImage;
static_assert(kStagesImage >= kStages8 && kStagesImage >= kStagesDual, "stage barriers");
constexpr int kExpanderWarps = 4;                // warps 4-7 (int8 -> fp16 stage expansion), one arrival each
constexpr int kBarBFull = 0;                     // [kMaxStages] fp16 stage ready for the MMA
constexpr int kBarBEmpty = kBarBFull + kMaxStages;  // [kMaxStages] MMAs reading the stage done
constexpr int kBarI8Full = kBarBEmpty + kMaxStages;  // [kI8Slots] int8 tile landed
constexpr int kBarI8Empty = kBarI8Full + kI8Slots;   // [kI8Slots] expanders done reading it
constexpr int kAccBufs = 3;                      // accumulator buffers in TMEM
constexpr int kBarAFull = kBarI8Empty + kI8Slots;  // A operand of the unit written to TMEM
constexpr int kBarAEmpty = kBarAFull + 1;        // MMAs of the unit done with A
constexpr int kBarAccFull = kBarAEmpty + 1;      // [kAccBufs] accumulator ready
constexpr int kBarAccEmpty = kBarAccFull + kAccBufs;  // [kAccBufs] accumulator drained (four quarters loaded)
constexpr int kBarRhoFull = kBarAccEmpty + kAccBufs;  // [4] per-unit row de-scale written
constexpr int kBarMFull = kBarRhoFull + 4;       // [2] groups 1.. partials staged for the merge
constexpr int kBarMEmpty = kBarMFull + 2;        // [2] group 0 consumed them
constexpr int kBarMmaDone = kBarMEmpty + 2;      // all MMAs retired (teardown)
constexpr int kBarCtabFull = kBarMmaDone + 1;    // [4] class table of a tile in log2 units
constexpr int kBarCtabEmpty = kBarCtabFull + 4;  // [4] all epilogue groups are done with it
constexpr int kBarCtabRaw = kBarCtabEmpty + 4;   // [4] (scale, bias) of a tile landed
constexpr int kBarStageFull = kBarCtabRaw + 4;   // f32 feature rows of the next unit landed
constexpr int kBarStageRead = kBarStageFull + 1;  // converters done reading the staged rows
constexpr int kNumBars = kBarStageRead + 1;
static_assert(kNumBars <= 48, "barrier area");

// TMEM columns: A operand [0,128) (hi and lo fp16 parts, 2 per column), accumulators
// [128,256), [256,384), [384,512).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = 0;
constexpr uint32_t kTmemAcc = 128;

constexpr uint32_t kSleepHintNs = 20000;  // longest a waiting thread stays suspended per try

struct Unit {
    int mb, sp, c0, c1;
};

// Units: row blocks [0, whole_units) with the whole class range (unit u = row block u; the
// plan makes whole_units a multiple of the grid, so they fill whole waves in row-block order),
// then every later row block split into n_splits class ranges (unit whole_units + v = split
// v % n_splits of row block whole_units + v / n_splits). A CTA takes units blockIdx.x,
// blockIdx.x + gridDim.x, ...
__device__ __forceinline__ bool unit_exists(int u, const HeadParams& p) {
    return u < p.whole_units + (p.n_mblocks - p.whole_units) * p.n_splits;
}

__device__ __forceinline__ Unit unit_of(int u, const HeadParams& p) {
    Unit U;
    if (u < p.whole_units) {
        U.mb = u;
        U.sp = 0;
        U.c0 = 0;
        U.c1 = p.n_chunks;
        return U;
    }
    const int v = u - p.whole_units;
    const int blk = v / p.n_splits;
    U.mb = p.whole_units + blk;
    U.sp = v - blk * p.n_splits;
    U.c0 = U.sp * p.chunks_per_split;
    U.c1 = min(U.c0 + p.chunks_per_split, p.n_chunks);
    return U;
}

// Bounded mbarrier wait. Gives up when another role has aborted or after timeout_ns, in
// which case it raises the CTA abort flag and the device status; every role then leaves
// its loop and the kernel tears down normally (TMEM freed, copies and MMAs drained).
__device__ __noinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                           const HeadParams& p, int where) {
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, kSleepHintNs)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > p.timeout_ns) {
            *abort_flag = 1u;
            atomicOr(p.status, kDevTimeout);
            atomicExch(p.status + 1, where);
            return false;
        }
    }
}

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                         const HeadParams& p, int where) {
    if (mbar_try_wait(bar, parity)) return true;  // common case inline: no call on the hot path
    return wait_bar_slow(bar, parity, abort_flag, p, where);
}

// Teardown wait: bounded by time only (used to drain work that is already in flight).
__device__ __noinline__ void drain_bar(uint32_t bar, uint32_t parity, const HeadParams& p) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait_sleep(bar, parity, kSleepHintNs)) {
        if (globaltimer_ns() - t0 > p.timeout_ns) {
            atomicOr(p.status, kDevTimeout);
            return;
        }
    }
}

// One fp16 element of the A operand for MMA K-step `step`, slot j (0..15), of a row whose
// f32 values are `arow` scaled by `rs` (a power of two). Steps [0, hi_steps) hold the high
// part, steps [hi_steps, hi_steps + lo_steps) the low part; with a merged tail the last
// high step holds hi(16T..16T+7) in slots 0..7 and lo(16T..16T+7) in slots 8..15 (the
// weight tile repeats q[16T..16T+7] in the matching K slots).
__device__ __forceinline__ __half a_part(const float* arow, long long stride, bool valid, int k, float rs, int step,
                                         int j, int hi_steps, int merged) {
    int kk;
    bool want_lo;
    if (step < hi_steps) {
        if (merged && step == hi_steps - 1 && j >= 8) {
            kk = 16 * step + j - 8;
            want_lo = true;
        } else {
            kk = 16 * step + j;
            want_lo = false;
        }
    } else {
        kk = 16 * (step - hi_steps) + j;
        want_lo = true;
    }
    if (!valid || kk >= k) return __float2half_rn(0.0f);
    const float x = __ldg(arow + (long long)kk * stride) * rs;
    const __half h = __float2half_rn(x);
    if (!want_lo) return h;
    return __float2half_rn(x - __half2float(h));
}

// 2^x for x <= 0 on the FMA pipe, two lanes at once: x = j + f with j = rint(x) (magic-number
// rounding) and f in [-1/2, 1/2]; 2^f from a degree-5 polynomial fitted for minimax relative
// error on that interval (max 2.2e-7 in f32 Horner form, like ex2.approx); 2^j added to the
// exponent field. x is clamped at -126 so the result stays a normal number (or ~1e-38).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x.x = fmaxf(x.x, -126.0f);
    x.y = fmaxf(x.y, -126.0f);
    const float2 magic = make_float2(12582912.0f, 12582912.0f);  // 1.5 * 2^23
    const float2 r = __fadd2_rn(x, magic);
    const float2 j = __fadd2_rn(r, make_float2(-12582912.0f, -12582912.0f));
    const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), x);
    float2 p = make_float2(1.3276457e-3f, 1.3276457e-3f);
    p = __ffma2_rn(p, f, make_float2(9.6755419e-3f, 9.6755419e-3f));
    p = __ffma2_rn(p, f, make_float2(5.5507135e-2f, 5.5507135e-2f));
    p = __ffma2_rn(p, f, make_float2(2.4022120e-1f, 2.4022120e-1f));
    p = __ffma2_rn(p, f, make_float2(6.9314694e-1f, 6.9314694e-1f));
    p = __ffma2_rn(p, f, make_float2(1.0000001f, 1.0000001f));
    // low bits of r hold j (two's complement); (r << 23) adds j to the exponent of p
    const uint32_t bx = __float_as_uint(p.x) + (__float_as_uint(r.x) << 23);
    const uint32_t by = __float_as_uint(p.y) + (__float_as_uint(r.y) << 23);
    return make_float2(__uint_as_float(bx), __uint_as_float(by));
}

// Two int8 weights stored as bytes b = q + 128 (selected from `w` by `sel`, a byte-permute
// selector placing them in bytes 0 and 2) -> two fp16 values q: 0x64 above each byte gives
// fp16 1024 + b, and subtracting 1152 leaves q exactly (all integers here are exact in fp16).
__device__ __forceinline__ uint32_t q8_to_f16x2(uint32_t w, uint32_t sel) {
    uint32_t h;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(h) : "r"(w), "r"(0x64646464u), "r"(sel));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(h) : "r"(0x64806480u));  // 0x6480 = fp16 1152
    return h;
}

// Order-preserving map of a (non-NaN) f32 onto u32: a < b  <=>  ord(a) < ord(b).
__device__ __forceinline__ uint32_t f32_ord(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Inverse of f32_ord.
__device__ __forceinline__ float ord_f32(uint32_t o) {
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

// Per-row state of one epilogue group over a work unit.
//   off, sum : sum = sum of 2^(t - off) over every column seen. off = 0 is the absolute
//              mode, kept while the row's max lies in [kAbsLo, kAbsHi]: there 2^t neither
//              overflows (18,816 terms <= 2^115) nor loses a term that matters (those below
//              2^-126 are < 2^-66 of the max), so no per-column offset is subtracted.
//              Otherwise off is the running max and the sum is rescaled when it rises.
//   best, idx: max and first argmax over the columns whose quarter reached the row's shared
//              threshold (see fused_quarter); the group that holds the unit's maximum always
//              tracks it, so the unit's (max, argmax) is the best of the groups' (best, idx).
//   thr      : last value of the shared threshold this thread read (never above it).
struct RowState {
    float off, sum, best;
    int idx;
    float thr;
};
constexpr float kAbsLo = -60.0f, kAbsHi = 100.0f;

// 32 accumulator columns of one row: t = D*c + e (the logit in log2 units), then the online
// update of `st`. In the relative mode the exps are taken against the running max from
// before these columns (so they need not wait for this quarter's max); the sum is rescaled
// once if the max rose, and recomputed exactly in the rare case that it rose by more than 64
// (2^64 bounds every term, so nothing overflows). `cs`/`es` are the shared-memory class
// table entries of these columns (shared-window addresses; warp-uniform, broadcast loads).
//
// First-argmax search: a quarter is searched only when its max beats the group's own best
// AND reaches the row's threshold `rowmax` - the largest best any epilogue group has
// published for this row in this unit (a 64-bit word: unit tag above, f32_ord(best) below;
// a word with another tag counts as no threshold). The threshold never exceeds the unit's
// true maximum, so the quarter that holds the first maximum is always searched, while the
// other groups stop searching quarters that cannot win.
// First index i in [B, B+8) with t[i] == q (the caller knows one exists).
template <int B>
__device__ __forceinline__ int first_in_octant(const float* t, float q) {
    int f = B + 7;
#pragma unroll
    for (int i = B + 6; i >= B; --i)
        if (t[i] == q) f = i;
    return f;
}

// t = D*c + e for four columns i..i+3 (the class table entries are warp-uniform broadcast
// loads from shared memory).
template <bool SCALED>
__device__ __forceinline__ void quarter_t4(const uint32_t* v, uint32_t cs, uint32_t es, float rho, int i, float* t) {
    const float4 c4 = lds128(cs + 4u * i);
    const float4 e4 = lds128(es + 4u * i);
    float2 x01 = make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1]));
    float2 x23 = make_float2(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
    if (SCALED) {
        x01 = __fmul2_rn(x01, make_float2(rho, rho));
        x23 = __fmul2_rn(x23, make_float2(rho, rho));
    }
    const float2 t01 = __ffma2_rn(x01, make_float2(c4.x, c4.y), make_float2(e4.x, e4.y));
    const float2 t23 = __ffma2_rn(x23, make_float2(c4.z, c4.w), make_float2(e4.z, e4.w));
    t[i] = t01.x;
    t[i + 1] = t01.y;
    t[i + 2] = t23.x;
    t[i + 3] = t23.y;
}

// 2^(t[i] - off), 2^(t[i+1] - off) (off = 0: no subtraction) added to acc; pairs below
// NPOLY go to the FMA-pipe polynomial instead of the MUFU.
template <int NPOLY, bool REL>
__device__ __forceinline__ void quarter_exp2(const float* t, int i, float2 nm, float2& acc) {
    float2 x = make_float2(t[i], t[i + 1]);
    if (REL) x = __fadd2_rn(x, nm);
    float2 e;
    if ((i >> 1) < NPOLY)
        e = exp2_poly2(x);
    else
        e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
    acc = __fadd2_rn(acc, e);
}

// Maxima of the quarter's four 8-column octants (kept for the first-argmax search, which then
// scans one octant instead of 32 columns).
__device__ __forceinline__ void quarter_octants(const float* t, float* oct) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
        oct[j] = max3f(max3f(t[8 * j], t[8 * j + 1], t[8 * j + 2]), max3f(t[8 * j + 3], t[8 * j + 4], t[8 * j + 5]),
                       fmaxf(t[8 * j + 6], t[8 * j + 7]));
}

// The t values, their exps and the octant maxima of a quarter whose offset is already known,
// as one straight-line block: the compiler can then interleave the MUFU exps with the shared
// loads, FMAs and max tree, so each warp keeps the MUFU fed instead of alternating an
// ALU phase with a burst of 32 exps.
template <bool SCALED, int NPOLY, bool REL>
__device__ __forceinline__ void quarter_known_offset(const uint32_t* v, uint32_t cs, uint32_t es, float rho, float off,
                                                     float* t, float* oct, float2& acc) {
    const float2 nm = make_float2(-off, -off);
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
        quarter_t4<SCALED>(v, cs, es, rho, i, t);
        quarter_exp2<NPOLY, REL>(t, i, nm, acc);
        quarter_exp2<NPOLY, REL>(t, i + 2, nm, acc);
    }
    quarter_octants(t, oct);
}

template <bool SCALED, int NPOLY, bool FIRST>
__device__ __forceinline__ void fused_quarter(const uint32_t* v, uint32_t cs, uint32_t es, int col0,
                                              float rho, uint32_t rowmax, uint32_t tag, RowState& st) {
    float t[32];
    float oct[4];
    float2 acc = make_float2(0.f, 0.f);
    float qmax;
    if constexpr (FIRST) {  // first columns of this row in the unit: the max picks the mode
#pragma unroll
        for (int i = 0; i < 32; i += 4) quarter_t4<SCALED>(v, cs, es, rho, i, t);
        quarter_octants(t, oct);
        qmax = max3f(oct[0], oct[1], fmaxf(oct[2], oct[3]));
        // (no early return for padded-only columns: every lane reaches the warp votes below)
        st.off = qmax == -CUDART_INF_F ? -CUDART_INF_F : (qmax >= kAbsLo && qmax <= kAbsHi) ? 0.0f : qmax;
        const float2 nm = make_float2(-st.off, -st.off);
        if (__all_sync(0xffffffffu, st.off == 0.0f)) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) quarter_exp2<NPOLY, false>(t, i, nm, acc);
        } else {
#pragma unroll
            for (int i = 0; i < 32; i += 2) quarter_exp2<NPOLY, true>(t, i, nm, acc);
        }
    } else {
        // The offset is known before this quarter, so the exps need not wait for the max
        // tree. A warp whose rows are all in the absolute mode skips the per-column subtraction.
        if (__all_sync(0xffffffffu, st.off == 0.0f))
            quarter_known_offset<SCALED, NPOLY, false>(v, cs, es, rho, 0.0f, t, oct, acc);
        else
            quarter_known_offset<SCALED, NPOLY, true>(v, cs, es, rho, st.off, t, oct, acc);
        qmax = max3f(oct[0], oct[1], fmaxf(oct[2], oct[3]));
    }
    float sq = acc.x + acc.y;
    // absolute mode: leave it only if the max passes kAbsHi; relative mode: rescale on a rise
    const float lim = st.off == 0.0f ? kAbsHi : st.off;
    if (FIRST && st.off == -CUDART_INF_F) {
        st.sum = 0.0f;  // padded classes only: nothing to add
    } else if (FIRST && st.off == 0.0f) {
        st.sum = sq;
    } else if (qmax > lim) {
        if (qmax - st.off > 64.0f) {  // exact recompute relative to the new max
            sq = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) sq += ex2_approx(t[i] - qmax);
            st.sum = (st.off == -CUDART_INF_F || FIRST ? 0.0f : st.sum * ex2_approx(st.off - qmax)) + sq;
        } else {
            st.sum = ((FIRST ? 0.0f : st.sum) + sq) * ex2_approx(st.off - qmax);
        }
        st.off = qmax;
    } else {
        st.sum = (FIRST ? 0.0f : st.sum) + sq;
    }
    if (qmax > st.best && qmax >= st.thr) {
        const unsigned long long w = lds_u64(rowmax);
        const uint32_t thr = (uint32_t)(w >> 32) == tag ? (uint32_t)w : 0u;
        st.thr = thr ? ord_f32(thr) : -CUDART_INF_F;
        const uint32_t qo = f32_ord(qmax);
        if (qo >= thr) {
            // first octant holding the maximum, then the first column of it within that octant
            int first;
            if (oct[0] == qmax)
                first = first_in_octant<0>(t, qmax);
            else if (oct[1] == qmax)
                first = first_in_octant<8>(t, qmax);
            else if (oct[2] == qmax)
                first = first_in_octant<16>(t, qmax);
            else
                first = first_in_octant<24>(t, qmax);
            st.best = qmax;
            st.idx = col0 + first;
            if (qo > thr) atom_max_shared_u64(rowmax, ((unsigned long long)tag << 32) | qo);
        }
    }
}

// Logits of 32 columns: dot * scale + bias; `cp` points at the columns' scales in the
// weight's class table, their biases sit 128 floats further.
template <bool SCALED>
__device__ __forceinline__ void logits_quarter(const uint32_t* v, const float* __restrict__ cp, int col0,
                                               float rho, float* __restrict__ out_row, int n) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float sc = __ldg(cp + i), bi = __ldg(cp + 128 + i);
        float x = __uint_as_float(v[i]);
        if (SCALED) x *= rho;
        if (col0 + i < n) out_row[col0 + i] = fmaf(x, sc, bi);
    }
}

// Merges two (max, sum of 2^(t - max), first argmax) triples (log2 units); ties keep the
// lower class index.
__device__ __forceinline__ void combine(float& m0, float& s0, int& i0, float m1, float s1, int i1) {
    const bool take1 = (m1 > m0) || (m1 == m0 && i1 < i0);
    const float M = take1 ? m1 : m0;
    float S = 0.f;
    if (m0 != -CUDART_INF_F) S += s0 * ex2_approx(m0 - M);
    if (m1 != -CUDART_INF_F) S += s1 * ex2_approx(m1 - M);
    i0 = take1 ? i1 : i0;
    m0 = M;
    s0 = S;
}

}  // namespace

// ------------------------------------------------------------------------- pack
// One warp per (padded) class row. Lane l holds K values l, l+32, l+64, l+96.
// Writes the class table (scale, bias) and the tiles, in one of two forms:
//  - fp16 image (the MMA's B operand as it sits in shared memory, one bulk copy per tile);
//  - int8 (compact): q + 128 as a byte (so the expander can build fp16(1024 + byte) by a byte
//    permute and subtract 1152), at image8_offset(row, K slot).
// K slots >= k hold q = 0, and with a merged tail the last hi step's upper 8 slots repeat its
// lower 8 (the low fp16 part of A rides there).
__global__ void __launch_bounds__(256) pack_kernel(const PackParams p) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= p.n_pad) return;
    const int j = warp;
    const bool real = j < p.n;
    float w[4];
    float max_abs = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int kk = lane + 32 * i;
        w[i] = (real && kk < p.k) ? p.w[(size_t)j * p.k + kk] : 0.0f;
        max_abs = fmaxf(max_abs, fabsf(w[i]));  // fmaxf ignores NaN, like f32::max
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) max_abs = fmaxf(max_abs, __shfl_xor_sync(0xffffffffu, max_abs, o));
    const float scale = max_abs > 1e-8f ? max_abs / 127.0f : 1.0f;  // IEEE division (no fast-math)
    const float inv_scale = 1.0f / scale;
    int q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float v = roundf(w[i] * inv_scale);  // half away from zero, like f32::round
        int qi;
        if (isnan(v))
            qi = 0;  // `NaN as i8` == 0
        else
            qi = (int)fminf(fmaxf(v, -127.0f), 127.0f);
        q[i] = real ? qi : 0;
    }
    const int tile = j >> 7, r = j & 127;
    if (lane == 0) {
        const float b = (real && p.bias) ? p.bias[j] : 0.0f;
        p.ctab[(size_t)tile * kCtabFloats + r] = real ? scale : 0.0f;
        p.ctab[(size_t)tile * kCtabFloats + kBlockN + r] = real ? b : -CUDART_INF_F;
    }
    if (p.compact) {
        // int8 tiles: lane l writes K slots 4l..4l+3 (one 32-bit word of one 16-byte chunk)
        uint32_t word = 0u;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int s = lane * 4 + t;  // K slot 0..127
            int src = s;
            if (p.merged_tail && s >= 16 * p.tail_step + 8 && s < 16 * p.tail_step + 16) src = s - 8;
            const bool ok = src < p.k;
            const int from = src & 31, reg = src >> 5;
            const int v0 = __shfl_sync(0xffffffffu, q[0], from);
            const int v1 = __shfl_sync(0xffffffffu, q[1], from);
            const int v2 = __shfl_sync(0xffffffffu, q[2], from);
            const int v3 = __shfl_sync(0xffffffffu, q[3], from);
            const int val = ok ? (reg == 0 ? v0 : reg == 1 ? v1 : reg == 2 ? v2 : v3) : 0;
            word |= (uint32_t)(val + 128) << (8 * t);
        }
        *reinterpret_cast<uint32_t*>(p.btiles + (size_t)tile * kTile8Bytes + image8_offset(r, lane * 4)) = word;
        return;
    }
    // fp16 image: tile j/128, row r = j%128, K slot s -> byte offset
    // (s/64)*16384 + r*128 + (((s%64)/8) ^ (r%8))*16 + (s%8)*2
    uint8_t* img = p.btiles + (size_t)tile * kTileBytes;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int s = lane * 4 + t;  // K slot 0..127
        int src = s;
        if (p.merged_tail && s >= 16 * p.tail_step + 8 && s < 16 * p.tail_step + 16) src = s - 8;
        const bool ok = src < p.k;
        const int from = src & 31, reg = src >> 5;
        const int v0 = __shfl_sync(0xffffffffu, q[0], from);
        const int v1 = __shfl_sync(0xffffffffu, q[1], from);
        const int v2 = __shfl_sync(0xffffffffu, q[2], from);
        const int v3 = __shfl_sync(0xffffffffu, q[3], from);
        const int val = reg == 0 ? v0 : reg == 1 ? v1 : reg == 2 ? v2 : v3;
        const __half h = __int2half_rn(ok ? val : 0);
        const uint32_t off = (uint32_t)(s >> 6) * 16384u + (uint32_t)r * 128u +
                             (uint32_t)((((s & 63) >> 3) ^ (r & 7)) << 4) + (uint32_t)(s & 7) * 2u;
        *reinterpret_cast<__half*>(img + off) = h;
    }
}

// ---------------------------------------------------------------- pack (FP32)
// The FP32 head (matmul_transposed_b, src/ops/matmul.rs:514-897, used when the engine does not
// quantise the head): no int8. Each class row is scaled by an exact power of two 2^sh so that
// max |w| lands in [2^14, 2^15), then split into fp16 hi = fp16(w 2^sh) and
// lo = fp16(w 2^sh - hi) (~22 significant bits); the tile holds the hi image followed by the lo
// image, and the class table carries 2^-sh in place of the int8 scale. One warp per class.
__global__ void __launch_bounds__(256) pack_f32_kernel(const PackParams p) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= p.n_pad) return;
    const int j = warp;
    const bool real = j < p.n;
    float w[4];
    float max_abs = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int kk = lane + 32 * i;
        w[i] = (real && kk < p.k) ? p.w[(size_t)j * p.k + kk] : 0.0f;
        max_abs = fmaxf(max_abs, fabsf(w[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) max_abs = fmaxf(max_abs, __shfl_xor_sync(0xffffffffu, max_abs, o));
    int sh = 0;
    if (max_abs > 0.0f && max_abs <= 3.4028235e38f) {
        const int e = (int)((__float_as_uint(max_abs) >> 23) & 0xFFu) - 127;  // floor(log2) for normals
        sh = min(max(14 - e, -126), 126);
    }
    const float up = __uint_as_float((uint32_t)(127 + sh) << 23);
    const float down = __uint_as_float((uint32_t)(127 - sh) << 23);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] *= up;  // exact: a power of two
    const int tile = j >> 7, r = j & 127;
    if (lane == 0) {
        const float b = (real && p.bias) ? p.bias[j] : 0.0f;
        p.ctab[(size_t)tile * kCtabFloats + r] = real ? down : 0.0f;
        p.ctab[(size_t)tile * kCtabFloats + kBlockN + r] = real ? b : -CUDART_INF_F;
    }
    uint8_t* img = p.btiles + (size_t)tile * (2 * kTileBytes);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int s = lane * 4 + t;  // K slot 0..127, same slot rule as the int8 image
        int src = s;
        if (p.merged_tail && s >= 16 * p.tail_step + 8 && s < 16 * p.tail_step + 16) src = s - 8;
        const bool ok = real && src < p.k;
        const int from = src & 31, reg = src >> 5;
        const float v0 = __shfl_sync(0xffffffffu, w[0], from);
        const float v1 = __shfl_sync(0xffffffffu, w[1], from);
        const float v2 = __shfl_sync(0xffffffffu, w[2], from);
        const float v3 = __shfl_sync(0xffffffffu, w[3], from);
        const float x = ok ? (reg == 0 ? v0 : reg == 1 ? v1 : reg == 2 ? v2 : v3) : 0.0f;
        const __half hi = __float2half_rn(x);
        const __half lo = __float2half_rn(x - __half2float(hi));
        const uint32_t off = (uint32_t)(s >> 6) * 16384u + (uint32_t)r * 128u +
                             (uint32_t)((((s & 63) >> 3) ^ (r & 7)) << 4) + (uint32_t)(s & 7) * 2u;
        *reinterpret_cast<__half*>(img + off) = hi;
        *reinterpret_cast<__half*>(img + kTileBytes + off) = lo;
    }
}

// Quantised weights: int8 tile number cc of this CTA, landed in slot cc % kI8Slots, is
// expanded into fp16 stage cc % kStages8 (the MMA's B operand, 128-byte swizzle) by the 128
// threads of warps 4-7. Each thread converts 8 chunks of 16 K slots: chunk i of warp w, lane l
// is row 16 i + 8 (w / 2) + l % 8, K chunk 4 (w % 2) + l / 8 (see image8_offset). A byte
// b = q + 128 becomes fp16 0x6400 | b = 1024 + b by a byte permute, minus 1152: exactly q.
// False when a wait gave up (uniform per warp).
__device__ __noinline__ bool expand_int8_tile(const HeadParams& p, uint32_t base, uint8_t* gbase, uint32_t cc, int w,
                                              int lane) {
    volatile uint32_t* abort_flag = reinterpret_cast<uint32_t*>(gbase + kOffMisc) + 1;
    const uint32_t bars = base + kOffBars;
    const uint32_t st = cc % (uint32_t)kStages8, i8 = cc % (uint32_t)kI8Slots;
    bool ok = wait_bar(bars + 8u * (kBarI8Full + i8), (cc / kI8Slots) & 1u, abort_flag, p, 14);
    ok = ok && wait_bar(bars + 8u * (kBarBEmpty + st), ((cc / kStages8) & 1u) ^ 1u, abort_flag, p, 15);
    if (!__all_sync(0xffffffffu, ok)) return false;
    const int rlow = lane & 7, j0 = 2 * (lane >> 3);
    const uint32_t src = base + kOffI8 + i8 * (uint32_t)kTile8Bytes + (uint32_t)(w * 32 + lane) * 16u;
    const uint32_t dst = base + kOffB + st * (uint32_t)kTileBytes + (uint32_t)(w & 1) * 16384u +
                         (uint32_t)(8 * (w >> 1) + rlow) * 128u;
    const uint32_t o0 = (uint32_t)((j0 ^ rlow) << 4), o1 = (uint32_t)(((j0 + 1) ^ rlow) << 4);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 b = lds128u(src + 2048u * (uint32_t)i);
        sts128u(dst + 2048u * (uint32_t)i + o0, make_uint4(q8_to_f16x2(b.x, 0x5140u), q8_to_f16x2(b.x, 0x7362u),
                                                          q8_to_f16x2(b.y, 0x5140u), q8_to_f16x2(b.y, 0x7362u)));
        sts128u(dst + 2048u * (uint32_t)i + o1, make_uint4(q8_to_f16x2(b.z, 0x5140u), q8_to_f16x2(b.z, 0x7362u),
                                                          q8_to_f16x2(b.w, 0x5140u), q8_to_f16x2(b.w, 0x7362u)));
    }
    // every thread orders its stage writes before the tensor core's (async-proxy) reads, the
    // warp synchronises, and one lane per warp releases the stage and the landing slot
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(bars + 8u * (kBarBFull + st));
        mbar_arrive(bars + 8u * (kBarI8Empty + i8));
    }
    return true;
}

// ----------------------------------------------------- converter / expander warps (4-7)
// A operand conversion per work unit and, for quantised weights, the int8 -> fp16 expansion of
// every weight tile. Kept out of line: its registers are allocated apart from the epilogue's.
__device__ __noinline__ void converter_warps(const HeadParams& p, uint32_t base, uint8_t* gbase, uint32_t tmem,
                                             int warp, int lane) {
    volatile uint32_t* abort_flag = reinterpret_cast<uint32_t*>(gbase + kOffMisc) + 1;
    float* rho_s = reinterpret_cast<float*>(gbase + kOffRho);
    uint32_t* qflag_s = reinterpret_cast<uint32_t*>(gbase + kOffQFlag);
    auto bar = [&](int i) -> uint32_t { return base + kOffBars + 8u * (uint32_t)i; };
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int steps = p.hi_steps + p.lo_steps;
    // Fast path (K % 4 == 0, 16-byte aligned features, and either the merged-tail layout of
    // K = 113..120 or a layout without a merged tail): the 128 feature rows of the next unit
    // are bulk-copied into shared memory while the current unit runs, so the A switch at a
    // unit boundary is a shared-memory -> TMEM conversion.
    const bool merged120 = p.hi_steps == 8 && p.lo_steps == 7 && p.merged_tail;
    const bool kt = p.a_t > 0;  // [batch][k][T] input: gathered by the converters themselves
    const bool staged = (merged120 || (!p.merged_tail && p.lo_steps == p.hi_steps)) && (p.k % 4) == 0 &&
                        (kt || (reinterpret_cast<uintptr_t>(p.a) & 15u) == 0);
    const bool bulk = staged && !kt;  // row-major: one bulk copy per unit
    const uint32_t lo_col = 8u * (uint32_t)p.hi_steps;  // first TMEM column of the low part
    const float* stage_g = reinterpret_cast<const float*>(gbase + kOffAStage);
    auto issue_stage = [&](int u) {  // one thread: rows of unit u -> staging buffer
        const Unit V = unit_of(u, p);
        const long long r0 = (long long)V.mb * kBlockM;
        const long long nrows = min((long long)kBlockM, p.m - r0);
        const uint32_t bytes = (uint32_t)(nrows * p.k * 4);
        mbar_arrive_expect_tx(bar(kBarStageFull), bytes);
        bulk_copy_g2s(base + kOffAStage, p.a + r0 * p.k, bytes, bar(kBarStageFull));
    };
    // [batch][k][T]: thread r gathers row r of unit u into the staging buffer (for one k the
    // 32 lanes of a warp read 32 consecutive timesteps: coalesced), while the previous unit runs.
    float* my_stage = const_cast<float*>(stage_g) + (size_t)r * p.k;
    auto gather_row = [&](int u) {
        const Unit V = unit_of(u, p);
        const long long row = (long long)V.mb * kBlockM + r;
        if (row >= p.m) return;
        const float* src = p.a + (row / p.a_t) * (long long)p.k * p.a_t + row % p.a_t;
        for (int kk = 0; kk < p.k; ++kk) my_stage[kk] = __ldg(src + (long long)kk * p.a_t);
    };
    uint32_t staged_issued = 0, staged_used = 0;
    if (bulk && r == 0 && unit_exists(blockIdx.x, p)) {
        issue_stage(blockIdx.x);
        staged_issued = 1;
    }
    if (staged && kt && unit_exists(blockIdx.x, p)) gather_row(blockIdx.x);
    const long long astride = kt ? p.a_t : 1;
    // A operand of unit u (the uc-th unit of this CTA) into TMEM; false when a wait gave up
    // (the caller then leaves its loop as a whole warp).
    auto convert_unit = [&](int u, uint32_t uc) -> bool {
        const Unit U = unit_of(u, p);
        const uint32_t slot = uc & 3u;
        const long long row = (long long)U.mb * kBlockM + r;
        const bool valid = row < p.m;
        const long long vrow = valid ? row : 0;
        const float* arow = staged ? stage_g + (size_t)r * p.k
                            : kt ? p.a + (vrow / p.a_t) * (long long)p.k * p.a_t + vrow % p.a_t
                                 : p.a + vrow * (long long)p.k;
        if (bulk) {
            if (!__all_sync(0xffffffffu, wait_bar(bar(kBarStageFull), uc & 1u, abort_flag, p, 12))) return false;
            staged_used = uc + 1;
        }
        float max_abs = 0.0f;
        if (valid) {
            if (staged) {
                for (int kk = 0; kk < p.k; kk += 4) {
                    const float4 x = lds128(smem_u32(arow + kk));
                    max_abs = fmaxf(max_abs, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
                }
            } else {
                for (int kk = 0; kk < p.k; ++kk) max_abs = fmaxf(max_abs, fabsf(__ldg(arow + (long long)kk * astride)));
            }
        }
        // fp16 holds the parts only below 65504: rows with max|a| >= 2^14 are scaled by a
        // power of two (exact) into [2^14, 2^15) and de-scaled in the epilogue.
        float rs = 1.0f, rho = 1.0f;
        if (max_abs >= 16384.0f && max_abs <= 3.4028235e38f) {
            const int e = (int)((__float_as_uint(max_abs) >> 23) & 0xFFu) - 127;
            rs = __uint_as_float((uint32_t)(127 + 14 - e) << 23);
            rho = __uint_as_float((uint32_t)(127 + e - 14) << 23);
        }
        const uint32_t need = __ballot_sync(0xffffffffu, rs != 1.0f);
        if (!__all_sync(0xffffffffu, wait_bar(bar(kBarAEmpty), (uc & 1u) ^ 1u, abort_flag, p, 5))) return false;
        tc_fence_after();
        const uint32_t a_t = tmem + lane_base + kTmemA;
        if (staged) {
            // pair p (K slots 2p, 2p+1): hi part -> column p; lo part -> column 8*hi_steps + p,
            // except the merged tail of K = 113..120 (p = 56..59 -> columns 60..63).
#pragma unroll 1
            for (int j = 0; j < p.hi_steps; ++j) {
                uint32_t hw[8], lw[8];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
                    const int kk = 16 * j + 8 * h;
                    if (valid && kk < p.k) {
                        x0 = lds128(smem_u32(arow + kk));
                        if (kk + 4 < p.k) x1 = lds128(smem_u32(arow + kk + 4));
                    }
                    const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        const float a0 = xs[2 * w] * rs, a1 = xs[2 * w + 1] * rs;
                        const __half2 hv = __floats2half2_rn(a0, a1);
                        const float2 hf = __half22float2(hv);
                        const __half2 lv = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
                        hw[4 * h + w] = *reinterpret_cast<const uint32_t*>(&hv);
                        lw[4 * h + w] = *reinterpret_cast<const uint32_t*>(&lv);
                    }
                }
                if (!merged120 || j < 7) {
                    tmem_st32x32b_x8(a_t + 8u * j, hw);
                    tmem_st32x32b_x8(a_t + lo_col + 8u * j, lw);
                } else {
                    const uint32_t h4[4] = {hw[0], hw[1], hw[2], hw[3]};
                    const uint32_t l4[4] = {lw[0], lw[1], lw[2], lw[3]};
                    tmem_st32x32b_x4(a_t + 56u, h4);
                    tmem_st32x32b_x4(a_t + 60u, l4);
                }
            }
            if (bulk) mbar_arrive(bar(kBarStageRead));
        } else {
            for (int g4 = 0; g4 * 4 < steps; ++g4) {
                uint32_t wv[32];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int step = g4 * 4 + t;
#pragma unroll
                    for (int w = 0; w < 8; ++w) {
                        uint32_t packed = 0u;
                        if (step < steps) {
                            const __half lo_h =
                                a_part(arow, astride, valid, p.k, rs, step, 2 * w, p.hi_steps, p.merged_tail);
                            const __half hi_h =
                                a_part(arow, astride, valid, p.k, rs, step, 2 * w + 1, p.hi_steps, p.merged_tail);
                            packed = (uint32_t)__half_as_ushort(lo_h) | ((uint32_t)__half_as_ushort(hi_h) << 16);
                        }
                        wv[t * 8 + w] = packed;
                    }
                }
                tmem_st32x32b_x32(a_t + (uint32_t)g4 * 32u, wv);
            }
        }
        tmem_st_wait();
        rho_s[slot * 128 + r] = rho;
        if (lane == 0) qflag_s[slot * 4 + q] = need;
        tc_fence_before();
        mbar_arrive(bar(kBarAFull));
        mbar_arrive(bar(kBarRhoFull + (int)slot));
        // next unit's rows into the staging buffer once every converter has read this one
        if (staged && kt && unit_exists(u + (int)gridDim.x, p)) gather_row(u + (int)gridDim.x);
        bool stop = false;
        if (bulk && r == 0 && unit_exists(u + (int)gridDim.x, p)) {
            if (wait_bar(bar(kBarStageRead), uc & 1u, abort_flag, p, 13)) {
                issue_stage(u + (int)gridDim.x);
                ++staged_issued;
            } else {
                stop = true;
            }
        }
        return !__any_sync(0xffffffffu, stop);  // leave as a whole warp
    };
    auto expand_tile = [&](uint32_t cc) -> bool { return expand_int8_tile(p, base, gbase, cc, warp & 3, lane); };
    if (!p.expand) {
        uint32_t uc = 0;
        for (int u = blockIdx.x; unit_exists(u, p); u += gridDim.x, ++uc)
            if (!convert_unit(u, uc)) break;
    } else {
        // One ordered sequence of tile expansions with each unit's A conversion inserted
        // right before the expansion of the unit's tile number kStages8 - 1: that expansion
        // waits for a stage the unit's own MMAs free (which need the unit's A), while the
        // conversion itself waits for the previous unit's MMAs (which need the expansions
        // before it). So no wait can depend on a later step of this sequence.
        int au = blockIdx.x;       // next unit whose A is converted
        uint32_t auc = 0, a_first = 0;  // its number within this CTA, its first tile number
        uint32_t cc = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && unit_exists(u, p); u += gridDim.x) {
            const Unit U = unit_of(u, p);
            for (int c = U.c0; ok && c < U.c1; ++c, ++cc) {
                if (unit_exists(au, p) && cc == a_first + (uint32_t)kStages8 - 1u) {
                    const Unit A = unit_of(au, p);
                    ok = convert_unit(au, auc);
                    a_first += (uint32_t)(A.c1 - A.c0);
                    au += gridDim.x;
                    ++auc;
                }
                ok = ok && expand_tile(cc);
            }
        }
        for (; ok && unit_exists(au, p); au += gridDim.x, ++auc) ok = convert_unit(au, auc);
    }
    // a staged copy still in flight must land before the CTA exits
    if (bulk && r == 0 && staged_issued > staged_used) drain_bar(bar(kBarStageFull), (staged_issued - 1) & 1u, p);
}

// ------------------------------------------------------------ epilogue warps (8-31)
template <bool EMIT_LOGITS, int NPOLY>
__device__ __noinline__ void epilogue_warps(const HeadParams& p, uint32_t base, uint8_t* gbase, uint32_t tmem,
                                            int warp, int lane) {
    volatile uint32_t* abort_flag = reinterpret_cast<uint32_t*>(gbase + kOffMisc) + 1;
    float* rho_s = reinterpret_cast<float*>(gbase + kOffRho);
    uint32_t* qflag_s = reinterpret_cast<uint32_t*>(gbase + kOffQFlag);
    float4* merge_s = reinterpret_cast<float4*>(gbase + kOffMerge);
    auto bar = [&](int i) -> uint32_t { return base + kOffBars + 8u * (uint32_t)i; };
    // ------------------------------------------------------------- epilogue
    // A group takes a 64-column half of a tile: two 32-column TMEM loads, each followed by
    // its math from registers; the accumulator goes back to the MMA issuer once both halves'
    // second quarters are loaded. One pair of waits, releases and loop steps serves 64
    // columns. Six groups give every SM sub-partition six independent warps of softmax work;
    // a group sees a different column subset of each row, which the online update and the
    // merge at the end of the unit do not mind.
    const int g = (warp - 8) >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t cc0 = 0, uc = 0;  // tiles before this unit, units so far
    bool ok = true;
    for (int u = blockIdx.x; ok && unit_exists(u, p); u += gridDim.x, ++uc) {
        const Unit U = unit_of(u, p);
        const uint32_t ntile = (uint32_t)(U.c1 - U.c0);
        const uint32_t slot = uc & 3u;
        const long long row = (long long)U.mb * kBlockM + r;
        RowState st{-CUDART_INF_F, 0.0f, -CUDART_INF_F, 0, -CUDART_INF_F};
        const uint32_t tag = uc + 1u;  // row thresholds of earlier units carry smaller tags
        const uint32_t rowmax = base + kOffRowMax + 8u * (uint32_t)r;
        if (!__all_sync(0xffffffffu, wait_bar(bar(kBarRhoFull + (int)slot), (uc >> 2) & 1u, abort_flag, p, 6))) break;
        const float rho = rho_s[slot * 128 + r];
        const bool scaled = qflag_s[slot * 4 + q] != 0u;
        // this group's halves of the unit: H = 2*(tile within the unit) + h, H % 6 == g, each
        // the two 32-column quarters 2h, 2h+1 of its tile, loaded and processed one after the
        // other (numbered from each unit's start, so a row's summation order depends only on
        // its unit's tile range, not on which CTA runs the unit or what it ran before).
        const uint32_t he = 2u * ntile;
        bool first = true;
        // Ring positions of this group's first tile in the unit (accumulator buffer and
        // class-table slot, with their phases); the group's next half lies kEpiGroups / 2 = 3
        // tiles further, so they then advance by increments: the buffer stays (3 buffers) and
        // its phase flips, the slot moves 3 on (4 slots) and its phase flips when it wraps.
        static_assert(kEpiGroups == 6 && kAccBufs == 3 && kCtabSlots == 4, "ring advance per half below");
        uint32_t cc = cc0 + ((uint32_t)g >> 1);
        const uint32_t buf = cc % kAccBufs;
        uint32_t aph = (cc / kAccBufs) & 1u;
        uint32_t cslot = cc % kCtabSlots, cph = (cc / kCtabSlots) & 1u;
        int c = U.c0 + (g >> 1);
        for (uint32_t H = (uint32_t)g; H < he;
             H += kEpiGroups, cc += 3u, c += 3, aph ^= 1u, cph ^= (cslot != 0u) ? 1u : 0u, cslot = (cslot + 3u) & 3u) {
            // both waits at once on the common path (class table and accumulator ready)
            const bool ready = EMIT_LOGITS ? mbar_try_wait(bar(kBarAccFull + (int)buf), aph)
                                           : mbar_try_wait2(bar(kBarCtabFull + (int)cslot), cph,
                                                            bar(kBarAccFull + (int)buf), aph);
            if (!__all_sync(0xffffffffu, ready)) {
                if (!EMIT_LOGITS &&
                    !__all_sync(0xffffffffu, wait_bar(bar(kBarCtabFull + (int)cslot), cph, abort_flag, p, 11))) {
                    ok = false;
                    break;
                }
                if (!__all_sync(0xffffffffu, wait_bar(bar(kBarAccFull + (int)buf), aph, abort_flag, p, 7))) {
                    ok = false;
                    break;
                }
            }
            tc_fence_after();
#pragma unroll
            for (uint32_t kk = 0; kk < 2u; ++kk) {
                const uint32_t k = 2u * (H & 1u) + kk;
                uint32_t v[32];
                tmem_ld32x32b_x32_wait(tmem + lane_base + kTmemAcc + buf * 128u + 32u * k, v);
                if (kk == 1u) {  // both quarters of the half are in registers: release the accumulator
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(kBarAccEmpty + (int)buf));
                }
                const int col0 = c * kBlockN + 32 * (int)k;
                if (EMIT_LOGITS) {
                    const float* cp = p.ctab + (size_t)c * 256 + 32 * k;
                    float* out_row = p.logits + (row < p.m ? row : 0) * (long long)p.n;
                    if (row < p.m) {
                        if (scaled) logits_quarter<true>(v, cp, col0, rho, out_row, p.n);
                        else logits_quarter<false>(v, cp, col0, rho, out_row, p.n);
                    }
                } else {
                    const uint32_t cs = base + kOffCtab + cslot * kCtabBytes + 4u * 32u * k;
                    if (first) {
                        if (scaled)
                            fused_quarter<true, NPOLY / 2, true>(v, cs, cs + 512u, col0, rho, rowmax, tag, st);
                        else
                            fused_quarter<false, NPOLY / 2, true>(v, cs, cs + 512u, col0, rho, rowmax, tag, st);
                    } else {
                        if (scaled)
                            fused_quarter<true, NPOLY / 2, false>(v, cs, cs + 512u, col0, rho, rowmax, tag, st);
                        else
                            fused_quarter<false, NPOLY / 2, false>(v, cs, cs + 512u, col0, rho, rowmax, tag, st);
                    }
                    first = false;
                }
            }
            if (!EMIT_LOGITS) {
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarCtabEmpty + (int)cslot));
            }
        }
        if (!ok) break;
        cc0 += ntile;
        if (!EMIT_LOGITS) {
            // Merge the groups' partial rows for this unit through shared memory.
            const uint32_t mb2 = uc & 1u;
            float4* mg = merge_s + mb2 * (kEpiGroups - 1) * 128;
            if (g != 0) {
                if (!__all_sync(0xffffffffu, wait_bar(bar(kBarMEmpty + (int)mb2), ((uc >> 1) & 1u) ^ 1u, abort_flag, p, 8)))
                    break;
                mg[(g - 1) * 128 + r] = make_float4(st.off, st.sum, st.best, __int_as_float(st.idx));
                mbar_arrive(bar(kBarMFull + (int)mb2));
            } else {
                if (!__all_sync(0xffffffffu, wait_bar(bar(kBarMFull + (int)mb2), (uc >> 1) & 1u, abort_flag, p, 9))) break;
                float4 o[kEpiGroups - 1];
#pragma unroll
                for (int j = 0; j < kEpiGroups - 1; ++j) o[j] = mg[j * 128 + r];
                mbar_arrive(bar(kBarMEmpty + (int)mb2));
                // Unit maximum = the largest tracked best (the group holding the maximum
                // always tracks it); the argmax comes from the group(s) whose best equals
                // it (ties: lower class index); each sum is rescaled from its own offset.
                float M = st.best;
#pragma unroll
                for (int j = 0; j < kEpiGroups - 1; ++j) M = fmaxf(M, o[j].z);
                float S = st.off != -CUDART_INF_F ? st.sum * ex2_approx(st.off - M) : 0.0f;
                int I = st.best == M ? st.idx : 0x7fffffff;
#pragma unroll
                for (int j = 0; j < kEpiGroups - 1; ++j) {
                    if (o[j].x != -CUDART_INF_F) S += o[j].y * ex2_approx(o[j].x - M);
                    if (o[j].z == M) I = min(I, __float_as_int(o[j].w));
                }
                if (I == 0x7fffffff) I = 0;  // no class at all (cannot happen for a real unit)
                if (row < p.m) {
                    if (U.mb < p.whole_units || p.n_splits == 1) {
                        p.idx[row] = I;
                        p.prob[row] = 1.0f / S;
                    } else {  // rows of the split row blocks, from row 128 whole_units on
                        const long long row0 = (long long)p.whole_units * kBlockM;
                        p.partial[(size_t)U.sp * (size_t)(p.m - row0) + (size_t)(row - row0)] =
                            make_float4(M, S, __int_as_float(I), 0.0f);
                    }
                }
            }
        }
    }
}

// -------------------------------------------------------------------- head
// Warp roles (one CTA per SM, persistent over work units = (row block, class range)):
//   warp 0      lane 0: weight-tile producer (TMA bulk copies into the smem ring)
//   warp 1      TMEM allocator; elected lane: MMA issuer
//   warp 2      lane 0 (fused variant): class-table producer (TMA bulk copies, 4-slot ring)
//   warp 3      idle
//   warps 4-7   A converters: f32 rows -> (hi, lo) fp16 parts in TMEM, one lane quadrant each
//   warps 8-31  epilogue groups 0-5 (4 warps each, lane quadrants 0-3); the 64-column
//               halves of a unit's accumulator tiles, numbered in order from the unit's
//               start, go round-robin to the groups: group g takes halves g, g+6, ...
template <bool EMIT_LOGITS, int NPOLY>
__global__ void __launch_bounds__(kHeadThreads, 1) head_kernel(const __grid_constant__ HeadParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t base = (raw_u32 + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw_u32);
    uint32_t* misc = reinterpret_cast<uint32_t*>(gbase + kOffMisc);
    volatile uint32_t* abort_flag = misc + 1;
    auto bar = [&](int i) -> uint32_t { return base + kOffBars + 8u * (uint32_t)i; };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            // int8 tiles: the expander warps fill a stage; otherwise one bulk copy (transaction bytes)
            mbar_init(bar(kBarBFull + s), p.expand ? kExpanderWarps : 1);
            mbar_init(bar(kBarBEmpty + s), 1);
        }
        for (int s = 0; s < kI8Slots; ++s) {
            mbar_init(bar(kBarI8Full + s), 1);
            mbar_init(bar(kBarI8Empty + s), kExpanderWarps);
        }
        mbar_init(bar(kBarAFull), 128);
        mbar_init(bar(kBarAEmpty), 1);
        mbar_init(bar(kBarStageFull), 1);
        mbar_init(bar(kBarStageRead), 128);
        for (int i = 0; i < kAccBufs; ++i) {
            mbar_init(bar(kBarAccFull + i), 1);
            mbar_init(bar(kBarAccEmpty + i), 8);  // one arrival per epilogue warp and half
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(kBarMFull + i), 128 * (kEpiGroups - 1));
            mbar_init(bar(kBarMEmpty + i), 128);
        }
        for (int i = 0; i < 4; ++i) {
            mbar_init(bar(kBarRhoFull + i), 128);
            mbar_init(bar(kBarCtabFull + i), 1);    // one lane of the class-table warp
            mbar_init(bar(kBarCtabEmpty + i), 8);  // one arrival per epilogue warp and half
            mbar_init(bar(kBarCtabRaw + i), 1);
        }
        mbar_init(bar(kBarMmaDone), 1);
        misc[1] = 0u;
        fence_mbar_init();
    }
    if (threadIdx.x < 128) {  // row thresholds start with tag 0: no unit has published yet
        reinterpret_cast<unsigned long long*>(gbase + kOffRowMax)[threadIdx.x] = 0ull;
    }
    if (warp == 1) {
        tmem_alloc(base + kOffMisc, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        // The whole warp runs the loop (uniform control flow); one elected lane issues.
        // fp16 image and FP32 weights: each tile (32 KB, or 64 KB for the FP32 (hi, lo) pair)
        // goes straight into an fp16 stage. int8 tiles: each 16 KB tile goes into a landing slot,
        // which the expander warps turn into an fp16 stage.
        const uint32_t ring = p.expand ? (uint32_t)kI8Slots : p.dual ? (uint32_t)kStagesDual : (uint32_t)kStagesImage;
        const uint32_t tile_bytes = p.expand ? (uint32_t)kTile8Bytes : p.dual ? 2u * kTileBytes : (uint32_t)kTileBytes;
        const uint32_t dst0 = base + (p.expand ? kOffI8 : kOffB);
        const int bar_full = p.expand ? kBarI8Full : kBarBFull;
        const int bar_empty = p.expand ? kBarI8Empty : kBarBEmpty;
        uint32_t cc = 0, issued = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && unit_exists(u, p); u += gridDim.x) {
            const Unit U = unit_of(u, p);
            for (int c = U.c0; c < U.c1; ++c, ++cc) {
                const int s = (int)(cc % ring);
                ok = __all_sync(0xffffffffu,
                                wait_bar(bar(bar_empty + s), ((cc / ring) & 1u) ^ 1u, abort_flag, p, 1));
                if (!ok) break;
                if (p.debug_flags & kDebugStallProducer) continue;
                if (elect_one()) {
                    mbar_arrive_expect_tx(bar(bar_full + s), tile_bytes);
                    bulk_copy_g2s(dst0 + (uint32_t)s * tile_bytes, p.btiles + (size_t)c * tile_bytes, tile_bytes,
                                  bar(bar_full + s));
                }
                __syncwarp();
                issued = cc + 1;
            }
        }
        // Drain: the last copy issued into each slot must land before the CTA exits.
        for (uint32_t s = 0; s < ring && s < issued; ++s) {
            const uint32_t fills = (issued - 1 - s) / ring + 1;
            drain_bar(bar(bar_full + (int)s), (fills - 1) & 1u, p);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        // Whole warp, uniform control flow; elect.sync inside the issue sequences.
        const uint32_t idesc = idesc_f16_f32(128, 128);
        const int steps = p.hi_steps + p.lo_steps;
        const bool k120 = p.hi_steps == 8 && p.lo_steps == 7 && p.merged_tail;  // K in 113..120
        const bool k80 = p.hi_steps == 5 && p.lo_steps == 5 && !p.merged_tail;  // K in 73..80
        // Per-step B descriptor offsets (16-byte units, added to the stage's descriptor).
        uint32_t boff[16];
#pragma unroll
        for (int step = 0; step < 16; ++step) {
            const int kc = step < p.hi_steps ? step : step - p.hi_steps;
            boff[step] = ((uint32_t)(kc >> 2) * 16384u + (uint32_t)(kc & 3) * 32u) >> 4;
        }
        const uint32_t tile_bytes = p.dual ? 2u * kTileBytes : kTileBytes;  // one fp16 stage
        const uint32_t nst = p.dual ? (uint32_t)kStagesDual : p.expand ? (uint32_t)kStages8 : (uint32_t)kStagesImage;
        // Ring positions (weight stage s, accumulator buf) and their phase bits advance by
        // increments and the stage descriptor by addition: this loop is the tensor core's
        // only feed, and a division-based position costs it a dependent integer-divide
        // sequence per tile. Adding to the descriptor's 14-bit start-address field (address
        // / 16) cannot carry out of it: shared-window addresses stay below 256 KB.
        const uint64_t bdesc_ring = smem_desc_k_sw128(base + kOffB);
        const uint32_t stage_desc = tile_bytes >> 4;
        const uint32_t a_tmem = tmem + kTmemA;
        uint32_t s = 0, sph = 0, buf = 0, aph = 0, uc = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && unit_exists(u, p); u += gridDim.x, ++uc) {
            const Unit U = unit_of(u, p);
            ok = __all_sync(0xffffffffu, wait_bar(bar(kBarAFull), uc & 1u, abort_flag, p, 2));
            if (!ok) break;
            tc_fence_after();
            for (int c = U.c0; c < U.c1; ++c) {
                // both waits at once on the common path (stage and accumulator ready)
                bool w = mbar_try_wait2(bar(kBarBFull + (int)s), sph, bar(kBarAccEmpty + (int)buf), aph ^ 1u);
                if (!__all_sync(0xffffffffu, w)) {
                    w = wait_bar(bar(kBarBFull + (int)s), sph, abort_flag, p, 3);
                    w = w && wait_bar(bar(kBarAccEmpty + (int)buf), aph ^ 1u, abort_flag, p, 4);
                }
                ok = __all_sync(0xffffffffu, w);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + kTmemAcc + buf * 128u;
                const uint64_t bdesc0 = bdesc_ring + (uint64_t)(s * stage_desc);
                if (p.dual) {
                    if (k120) {
                        mma_tile_k120_dual_warp(d_tmem, a_tmem, bdesc0, idesc, bar(kBarBEmpty + s),
                                                bar(kBarAccFull + (int)buf));
                    } else {
                        // A_hi.W_hi + A_lo.W_hi, then A_hi.W_lo (lo image 32 KB further)
#pragma unroll
                        for (int step = 0; step < 16; ++step) {
                            if (step < steps)
                                mma_f16_ts_warp(d_tmem, a_tmem + (uint32_t)step * 8u, bdesc0 + boff[step], idesc,
                                                step > 0 ? 1u : 0u);
                        }
#pragma unroll
                        for (int step = 0; step < 8; ++step) {
                            if (step < p.hi_steps)
                                mma_f16_ts_warp(d_tmem, a_tmem + (uint32_t)step * 8u,
                                                bdesc0 + (kTileBytes >> 4) + boff[step], idesc, 1u);
                        }
                        mma_commit_warp(bar(kBarBEmpty + s));
                        mma_commit_warp(bar(kBarAccFull + (int)buf));
                    }
                } else if (k120) {
                    mma_tile_k120_warp(d_tmem, a_tmem, bdesc0, idesc, bar(kBarBEmpty + s), bar(kBarAccFull + (int)buf));
                } else if (k80) {
                    mma_tile_k80_warp(d_tmem, a_tmem, bdesc0, idesc, bar(kBarBEmpty + s), bar(kBarAccFull + (int)buf));
                } else {
#pragma unroll
                    for (int step = 0; step < 16; ++step) {
                        if (step < steps)
                            mma_f16_ts_warp(d_tmem, a_tmem + (uint32_t)step * 8u, bdesc0 + boff[step], idesc,
                                            step > 0 ? 1u : 0u);
                    }
                    mma_commit_warp(bar(kBarBEmpty + s));
                    mma_commit_warp(bar(kBarAccFull + (int)buf));
                }
                if (++s == nst) {
                    s = 0u;
                    sph ^= 1u;
                }
                if (++buf == (uint32_t)kAccBufs) {
                    buf = 0u;
                    aph ^= 1u;
                }
            }
            if (!ok) break;
            mma_commit_warp(bar(kBarAEmpty));
        }
        mma_commit_warp(bar(kBarMmaDone));
        drain_bar(bar(kBarMmaDone), 0u, p);
    } else if (warp == 2) {
        // ---------------------------------------------------- class-table producer
        // Per tile: the weight's (scale[128], bias[128]) land in a ring slot by one bulk copy,
        // then the warp converts them in place to log2 units, c = scale * log2(e) and
        // e = bias * log2(e), which the epilogue's t = D * c + e needs.
        if (!EMIT_LOGITS) {
            uint32_t cc = 0, pending = 0;  // pending: 1 + slot of a copy not yet seen landing
            bool ok = true;
            for (int u = blockIdx.x; ok && unit_exists(u, p); u += gridDim.x) {
                const Unit U = unit_of(u, p);
                for (int c = U.c0; c < U.c1; ++c, ++cc) {
                    const uint32_t slot = cc % kCtabSlots;
                    const uint32_t ph = (cc / kCtabSlots) & 1u;
                    ok = __all_sync(0xffffffffu, wait_bar(bar(kBarCtabEmpty + (int)slot), ph ^ 1u, abort_flag, p, 10));
                    if (!ok) break;
                    const uint32_t dst = base + kOffCtab + slot * kCtabBytes;
                    if (elect_one()) {
                        mbar_arrive_expect_tx(bar(kBarCtabRaw + (int)slot), kCtabBytes);
                        bulk_copy_g2s(dst, p.ctab + (size_t)c * kCtabFloats, kCtabBytes, bar(kBarCtabRaw + (int)slot));
                    }
                    __syncwarp();
                    pending = slot + 1u;
                    ok = __all_sync(0xffffffffu, wait_bar(bar(kBarCtabRaw + (int)slot), ph, abort_flag, p, 16));
                    if (!ok) break;
                    pending = 0u;
                    float4 sc = lds128(dst + 16u * lane);
                    float4 bi = lds128(dst + 512u + 16u * lane);
                    sc = make_float4(sc.x * kLog2e, sc.y * kLog2e, sc.z * kLog2e, sc.w * kLog2e);
                    bi = make_float4(bi.x * kLog2e, bi.y * kLog2e, bi.z * kLog2e, bi.w * kLog2e);
                    sts128(dst + 16u * lane, sc);
                    sts128(dst + 512u + 16u * lane, bi);
                    // the slot is next overwritten by a bulk copy (async proxy); every lane's
                    // writes are ordered before the one arrival by the warp synchronisation
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(kBarCtabFull + (int)slot));
                }
            }
            if (pending) {  // a copy in flight when another role aborted must land before exit
                const uint32_t slot = pending - 1u;
                drain_bar(bar(kBarCtabRaw + (int)slot), ((cc / kCtabSlots) & 1u), p);
            }
        }
    } else if (warp >= 4 && warp < 8) {
        converter_warps(p, base, gbase, tmem, warp, lane);
    } else if (warp >= 8) {
        epilogue_warps<EMIT_LOGITS, NPOLY>(p, base, gbase, tmem, warp, lane);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ------------------------------------------------------------------- merge
__global__ void __launch_bounds__(256) merge_kernel(const float4* __restrict__ partial, int n_splits, long long m,
                                                    int32_t* __restrict__ idx, float* __restrict__ prob) {
    const long long row = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= m) return;
    float M = -CUDART_INF_F, S = 0.0f;
    int I = 0;
    for (int s = 0; s < n_splits; ++s) {
        const float4 v = partial[(size_t)s * (size_t)m + (size_t)row];
        combine(M, S, I, v.x, v.y, __float_as_int(v.z));
    }
    idx[row] = I;
    prob[row] = 1.0f / S;
}

// ------------------------------------------------------------------ launchers
size_t head_smem_bytes() { return kSmemBytes; }

template <bool L, int NP>
static cudaError_t set_smem_attr() {
    return cudaFuncSetAttribute(head_kernel<L, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
}

cudaError_t head_kernel_setup() {
    cudaError_t e;
    if ((e = set_smem_attr<true, 0>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<false, 0>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<false, 2>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<false, 4>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<false, 6>()) != cudaSuccess) return e;
    return set_smem_attr<false, 8>();
}

cudaError_t launch_pack(const PackParams& p, cudaStream_t stream) {
    const int threads = 256;
    const long long total = (long long)p.n_pad * 32;
    const int blocks = (int)((total + threads - 1) / threads);
    if (p.f32)
        pack_f32_kernel<<<blocks, threads, 0, stream>>>(p);
    else
        pack_kernel<<<blocks, threads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_head(const HeadParams& p, bool emit_logits, int grid, cudaStream_t stream) {
    if (emit_logits) {
        head_kernel<true, 0><<<grid, kHeadThreads, kSmemBytes, stream>>>(p);
    } else {
        switch (p.poly_pairs) {
            case 0: head_kernel<false, 0><<<grid, kHeadThreads, kSmemBytes, stream>>>(p); break;
            case 2: head_kernel<false, 2><<<grid, kHeadThreads, kSmemBytes, stream>>>(p); break;
            case 6: head_kernel<false, 6><<<grid, kHeadThreads, kSmemBytes, stream>>>(p); break;
            case 8: head_kernel<false, 8><<<grid, kHeadThreads, kSmemBytes, stream>>>(p); break;
            default: head_kernel<false, 4><<<grid, kHeadThreads, kSmemBytes, stream>>>(p); break;
        }
    }
    return cudaGetLastError();
}

cudaError_t launch_merge(const float4* partial, int n_splits, long long m, int32_t* idx, float* prob,
                         cudaStream_t stream) {
    const int threads = 256;
    const int blocks = (int)((m + threads - 1) / threads);
    merge_kernel<<<blocks, threads, 0, stream>>>(partial, n_splits, m, idx, prob);
    return cudaGetLastError();
}

}  // namespace rh
