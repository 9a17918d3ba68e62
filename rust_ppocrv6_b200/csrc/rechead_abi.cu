// Host side of the C ABI declared in include/rechead.h: contexts (one stream, status word
// and scratch per device), packed weights, work planning, launches, multi-device sharding of
// line batches and the host CTC collapse. No CPU fallback exists: every compute entry point
// runs the sm_100a kernels of rechead_kernels.cu or fails.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "head_params.h"
#include "recpre_params.h"
#include "rechead.h"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

#define RH_CUDA(call)                                                                         \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess) return fail(RH_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() { release(); }  // the owner has made the right device current
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap && p) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 256));
        if (e == cudaSuccess) cap = std::max<size_t>(bytes, 256);
        return e;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
};

struct Slot {
    int device = 0;
    int sms = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t copy_stream = nullptr;  // host-to-device copies that overlap the kernels
    cudaEvent_t copied = nullptr;
    int* d_status = nullptr;
    int* h_status = nullptr;  // pinned copy of d_status, read back at the end of a call
    DevBuf a, idx, prob, out, partial;
    DevBuf lines, tok_off, tokens, scores;  // CTC collapse on the device
    DevBuf pre_rgb, pre_lines, pre_coords, pre_wts, pre_out;  // recognition preprocessing
    cudaEvent_t pre_done = nullptr;  // recorded after the last kernel that reads pre_lines/coords/wts
    cudaEvent_t part_done = nullptr;  // recorded after the last merge that reads `partial`
    std::mutex mu;
    int64_t launches = 0;
    // Frees everything, also on a context whose creation failed part-way.
    ~Slot() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        if (copy_stream) cudaStreamSynchronize(copy_stream);
        for (DevBuf* b : {&a, &idx, &prob, &out, &partial, &lines, &tok_off, &tokens, &scores, &pre_rgb, &pre_lines,
                          &pre_coords, &pre_wts, &pre_out})
            b->release();
        if (d_status) cudaFree(d_status);
        if (h_status) cudaFreeHost(h_status);
        if (copied) cudaEventDestroy(copied);
        if (pre_done) cudaEventDestroy(pre_done);
        if (part_done) cudaEventDestroy(part_done);
        if (copy_stream) cudaStreamDestroy(copy_stream);
        if (stream) cudaStreamDestroy(stream);
    }
};

struct Geometry {
    int n_chunks, hi_steps, lo_steps, merged, tail_step;
};

Geometry geometry(int64_t n, int64_t k) {
    Geometry g;
    g.n_chunks = (int)((n + rh::kBlockN - 1) / rh::kBlockN);
    const int k16 = (int)((k + 15) / 16);
    g.tail_step = k16 - 1;
    const int rem = (int)(k - 16 * g.tail_step);  // 1..16 values in the last K step
    g.merged = rem <= 8 ? 1 : 0;
    g.hi_steps = k16;
    g.lo_steps = g.merged ? k16 - 1 : k16;
    return g;
}

// Chooses the work units of a launch. As many full waves of whole row blocks (the whole class
// range, no merge) as the row blocks fill, then the remaining row blocks (fewer than the grid)
// split into as many class ranges as keep their last wave evenly loaded: cost = waves * (chunks
// per unit + per-unit overhead). Whole row blocks keep the number of units per CTA, and so of
// A-operand hand-overs between units, at its least (cfg2: 7 units per CTA instead of 13 with
// every row block split in two).
void plan(int64_t m, int n_chunks, int sms, int& n_mblocks, int& whole_units, int& n_splits, int& cps,
          int& grid) {
    n_mblocks = (int)((m + rh::kBlockM - 1) / rh::kBlockM);
    whole_units = (n_mblocks / sms) * sms;
    const int rest = n_mblocks - whole_units;
    double best = 1e300;
    n_splits = 1;
    cps = n_chunks;
    for (int s = 1; rest > 0 && s <= n_chunks; ++s) {
        const int c = (n_chunks + s - 1) / s;
        const int s_eff = (n_chunks + c - 1) / c;
        const long long units = (long long)rest * s_eff;
        const long long waves = (units + sms - 1) / sms;
        const double cost = (double)waves * (c + 2.0);
        if (cost < best - 1e-9) {
            best = cost;
            n_splits = s_eff;
            cps = c;
        }
    }
    const long long units = (long long)whole_units + (long long)rest * n_splits;
    grid = (int)std::min<long long>(units, sms);
}

// Rows whose idx/prob come through the split merge: those of the row blocks after the whole
// units, when they are split.
int64_t split_rows(const rh::HeadParams& p) {
    return p.n_splits > 1 ? p.m - (int64_t)p.whole_units * rh::kBlockM : 0;
}

std::vector<int> injected_fault_slots() {
    std::vector<int> v;
    const char* s = std::getenv("RH_FAULT_DEVICE");
    if (!s) return v;
    std::string str(s);
    size_t pos = 0;
    while (pos < str.size()) {
        size_t e = str.find(',', pos);
        if (e == std::string::npos) e = str.size();
        if (e > pos) v.push_back(std::atoi(str.substr(pos, e - pos).c_str()));
        pos = e + 1;
    }
    return v;
}

int poly_pairs_setting() {
    if (const char* s = std::getenv("RH_POLY_PAIRS")) return std::atoi(s);
    return rh::kDefaultPolyPairs;
}

}  // namespace

struct rh_ctx {
    std::vector<std::unique_ptr<Slot>> slots;
    unsigned long long timeout_ns = 2000000000ull;
};

struct rh_weight {
    int64_t n = 0, k = 0;
    bool f32 = false;      // FP32 head (rh_weight_pack_f32): hi/lo fp16 images, no int8
    bool compact = false;  // quantised, int8 tiles (rh_weight_pack_compact) instead of the fp16 image
    Geometry g{};
    // Per device: the weight tiles (quantised: the fp16 image of the MMA operand, 32 KB per 128
    // classes, or compact int8, 16 KB per 128 classes in the order the kernel expands them;
    // FP32: fp16 hi and lo images, 64 KB per 128 classes) and the class table (scale[128] then
    // bias[128] per tile). Nothing else stays on the device.
    struct Per {
        int device = 0;
        uint8_t* tiles = nullptr;
        float* ctab = nullptr;
    };
    std::vector<Per> per;
    std::vector<float> host_scales;  // per-class scale (int8 scale, or 2^-sh for FP32), to rebuild the table
    size_t tile_bytes() const {
        return f32 ? 2u * rh::kTileBytes : compact ? (size_t)rh::kTile8Bytes : (size_t)rh::kTileBytes;
    }
    // Frees every device copy, also for a weight whose packing failed part-way.
    ~rh_weight() {
        for (auto& p : per) {
            cudaSetDevice(p.device);
            cudaDeviceSynchronize();
            cudaFree(p.tiles);
            cudaFree(p.ctab);
        }
    }
};

namespace {

int check_ctx(rh_ctx* ctx) {
    if (!ctx || ctx->slots.empty()) return fail(RH_ERR_INVALID_ARG, "null or empty context");
    return RH_OK;
}

// Launch parameters of the head over rows [0, rows) of d_a (a_t > 0: the [batch][k][a_t]
// layout) with the planner's class-range split; `partial` is left for the caller to point at
// its split scratch. Every head launch path builds its parameters here.
rh::HeadParams head_params(rh_ctx* ctx, const rh_weight* w, const Slot& s, const rh_weight::Per& pw, const float* d_a,
                           int64_t rows, int64_t a_t, int32_t* d_idx, float* d_prob, float* d_logits, int& grid) {
    int n_mblocks, whole_units, n_splits, cps;
    plan(rows, w->g.n_chunks, s.sms, n_mblocks, whole_units, n_splits, cps, grid);
    rh::HeadParams p{};
    p.a = d_a;
    p.a_t = a_t;
    p.m = rows;
    p.k = (int)w->k;
    p.n = (int)w->n;
    p.n_chunks = w->g.n_chunks;
    p.hi_steps = w->g.hi_steps;
    p.lo_steps = w->g.lo_steps;
    p.merged_tail = w->g.merged;
    p.btiles = pw.tiles;
    p.dual = w->f32 ? 1 : 0;
    p.expand = w->compact ? 1 : 0;
    p.ctab = pw.ctab;
    p.poly_pairs = poly_pairs_setting();
    p.n_mblocks = n_mblocks;
    p.whole_units = whole_units;
    p.n_splits = n_splits;
    p.chunks_per_split = cps;
    p.idx = d_idx;
    p.prob = d_prob;
    p.logits = d_logits;
    p.partial = nullptr;
    p.status = s.d_status;
    p.timeout_ns = ctx->timeout_ns;
    p.debug_flags = 0;
    if (const char* dbg = std::getenv("RH_DEBUG_FLAGS")) p.debug_flags = std::atoi(dbg);
    return p;
}

// Launches the head, then (fused, class range split) the merge of the per-split partials in
// p.partial over the split row blocks' rows, on `stream`.
int launch_head_and_merge(Slot& s, const rh::HeadParams& p, bool emit_logits, int grid, cudaStream_t stream) {
    RH_CUDA(rh::launch_head(p, emit_logits, grid, stream));
    s.launches++;
    if (!emit_logits && split_rows(p) > 0) {
        const int64_t row0 = (int64_t)p.whole_units * rh::kBlockM;
        RH_CUDA(rh::launch_merge(p.partial, p.n_splits, split_rows(p), p.idx + row0, p.prob + row0, stream));
        s.launches++;
    }
    return RH_OK;
}

// Enqueues the head (and the split merge) for rows [0, rows) of d_a on `stream`.
int enqueue_head(rh_ctx* ctx, const rh_weight* w, Slot& s, const rh_weight::Per& pw, const float* d_a, int64_t rows,
                 int32_t* d_idx, float* d_prob, float* d_logits, bool emit_logits, cudaStream_t stream,
                 int64_t a_t = 0) {
    if (rows <= 0) return RH_OK;
    int grid;
    rh::HeadParams p = head_params(ctx, w, s, pw, d_a, rows, a_t, d_idx, d_prob, d_logits, grid);
    const bool split = !emit_logits && split_rows(p) > 0;
    if (split) {
        // The split scratch is the slot's: order this call after the previous merge that read
        // it (which may run on another caller stream), and let that merge finish before the
        // buffer is reallocated.
        if (!s.part_done) RH_CUDA(cudaEventCreateWithFlags(&s.part_done, cudaEventDisableTiming));
        const size_t need = (size_t)p.n_splits * (size_t)split_rows(p) * sizeof(float4);
        if (need > s.partial.cap) RH_CUDA(cudaEventSynchronize(s.part_done));
        RH_CUDA(s.partial.ensure(need));
        RH_CUDA(cudaStreamWaitEvent(stream, s.part_done, 0));
        p.partial = static_cast<float4*>(s.partial.p);
    }
    if (int rc = launch_head_and_merge(s, p, emit_logits, grid, stream)) return rc;
    if (split) RH_CUDA(cudaEventRecord(s.part_done, stream));
    return RH_OK;
}

// A non-zero device status word `st` (copied back from s.d_status) as an error; clears it.
int status_error(Slot& s, const int* st) {
    if (st[0] != 0) {
        RH_CUDA(cudaMemsetAsync(s.d_status, 0, 2 * sizeof(int), s.stream));
        RH_CUDA(cudaStreamSynchronize(s.stream));
        if (st[0] & rh::kDevTimeout)
            return fail(RH_ERR_TIMEOUT, "device wait timed out (site " + std::to_string(st[1]) +
                                            "); the kernel gave up and the context is still usable");
        return fail(RH_ERR_CUDA, "device status " + std::to_string(st[0]));
    }
    return RH_OK;
}

int read_status(Slot& s) {
    int st[2] = {0, 0};
    RH_CUDA(cudaMemcpyAsync(st, s.d_status, sizeof(st), cudaMemcpyDeviceToHost, s.stream));
    RH_CUDA(cudaStreamSynchronize(s.stream));
    return status_error(s, st);
}

// Waits for the work queued on the slot's stream and checks the device status, whose copy back
// is queued on the same stream first: one synchronisation at the end of a call, not two.
int sync_and_check(Slot& s) {
    RH_CUDA(cudaMemcpyAsync(s.h_status, s.d_status, 2 * sizeof(int), cudaMemcpyDeviceToHost, s.stream));
    RH_CUDA(cudaStreamSynchronize(s.stream));
    const int st[2] = {s.h_status[0], s.h_status[1]};
    return status_error(s, st);
}

const rh_weight::Per* weight_on(const rh_weight* w, int device) {
    for (const auto& p : w->per)
        if (p.device == device) return &p;
    return nullptr;
}

// Host-memory head on one slot: H2D rows, kernels, D2H results, synchronise, check status.
// The host-memory pass on one device; the caller holds s.mu. With idx == prob == logits ==
// nullptr the per-timestep (idx, prob) stay in s.idx / s.prob for a following device step.
int host_pass_locked(rh_ctx* ctx, const rh_weight* w, Slot& s, const float* a, int64_t rows, int32_t* idx,
                     float* prob, float* logits) {
    RH_CUDA(cudaSetDevice(s.device));
    const rh_weight::Per* pw = weight_on(w, s.device);
    if (!pw) return fail(RH_ERR_INVALID_ARG, "weight was not packed for this context's devices");
    const size_t a_bytes = (size_t)rows * (size_t)w->k * sizeof(float);
    RH_CUDA(s.a.ensure(a_bytes));
    const bool emit_logits = logits != nullptr;
    if (emit_logits) {
        RH_CUDA(cudaMemcpyAsync(s.a.p, a, a_bytes, cudaMemcpyHostToDevice, s.stream));
        const size_t o_bytes = (size_t)rows * (size_t)w->n * sizeof(float);
        RH_CUDA(s.out.ensure(o_bytes));
        int rc = enqueue_head(ctx, w, s, *pw, (const float*)s.a.p, rows, nullptr, nullptr, (float*)s.out.p, true,
                              s.stream);
        if (rc) return rc;
        RH_CUDA(cudaMemcpyAsync(logits, s.out.p, o_bytes, cudaMemcpyDeviceToHost, s.stream));
    } else {
        // Pipelined: pieces of one full wave of 128-row blocks. The copy of piece i+1 runs on the
        // copy stream while piece i computes; an event hands each piece to the compute stream.
        RH_CUDA(s.idx.ensure((size_t)rows * sizeof(int32_t)));
        RH_CUDA(s.prob.ensure((size_t)rows * sizeof(float)));
        const int64_t piece = (int64_t)s.sms * rh::kBlockM;
        const size_t row_bytes = (size_t)w->k * sizeof(float);
        for (int64_t r0 = 0; r0 < rows; r0 += piece) {
            const int64_t n = std::min(piece, rows - r0);
            const float* src = a + (size_t)r0 * (size_t)w->k;
            float* dst = (float*)s.a.p + (size_t)r0 * (size_t)w->k;
            RH_CUDA(cudaMemcpyAsync(dst, src, (size_t)n * row_bytes, cudaMemcpyHostToDevice, s.copy_stream));
            RH_CUDA(cudaEventRecord(s.copied, s.copy_stream));
            RH_CUDA(cudaStreamWaitEvent(s.stream, s.copied, 0));
            int rc = enqueue_head(ctx, w, s, *pw, dst, n, (int32_t*)s.idx.p + r0, (float*)s.prob.p + r0, nullptr,
                                  false, s.stream);
            if (rc) return rc;
        }
        // One copy of the results at the end: copies queued between the pieces would hold
        // each next piece's kernel behind them (measured: 1.43 -> 1.29 ms per cfg2 call).
        if (idx) {
            RH_CUDA(cudaMemcpyAsync(idx, s.idx.p, (size_t)rows * sizeof(int32_t), cudaMemcpyDeviceToHost, s.stream));
            RH_CUDA(cudaMemcpyAsync(prob, s.prob.p, (size_t)rows * sizeof(float), cudaMemcpyDeviceToHost, s.stream));
        }
    }
    return RH_OK;
}

int run_host_on_slot(rh_ctx* ctx, const rh_weight* w, int slot, const float* a, int64_t rows, int32_t* idx,
                     float* prob, float* logits) {
    if (rows <= 0) return RH_OK;
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    if (int rc = host_pass_locked(ctx, w, s, a, rows, idx, prob, logits)) return rc;
    return sync_and_check(s);
}

// The fused head then the CTC collapse on one device for lines [0, n_lines) of a shard whose
// rows start at a (line_offsets rebased so that line_offsets[0] == 0). tokens receives the
// shard's tokens back to back, token_offsets its n_lines + 1 offsets (from 0), scores one per
// line. Only the collapsed result comes back to the host.
int run_ctc_on_slot(rh_ctx* ctx, const rh_weight* w, int slot, const float* a, const int64_t* line_offsets,
                    int64_t n_lines, int32_t* tokens, int64_t* token_offsets, float* scores) {
    const int64_t rows = line_offsets[n_lines];
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    if (rows > 0) {
        if (int rc = host_pass_locked(ctx, w, s, a, rows, nullptr, nullptr, nullptr)) return rc;
    } else {
        RH_CUDA(cudaSetDevice(s.device));
        RH_CUDA(s.idx.ensure(sizeof(int32_t)));
        RH_CUDA(s.prob.ensure(sizeof(float)));
    }
    const size_t off_bytes = (size_t)(n_lines + 1) * sizeof(int64_t);
    RH_CUDA(s.lines.ensure(off_bytes));
    RH_CUDA(s.tok_off.ensure(off_bytes));
    RH_CUDA(s.tokens.ensure((size_t)std::max<int64_t>(rows, 1) * sizeof(int32_t)));
    RH_CUDA(s.scores.ensure((size_t)std::max<int64_t>(n_lines, 1) * sizeof(float)));
    RH_CUDA(cudaMemcpyAsync(s.lines.p, line_offsets, off_bytes, cudaMemcpyHostToDevice, s.stream));
    RH_CUDA(rh::launch_ctc_collapse((const int32_t*)s.idx.p, (const float*)s.prob.p, (const int64_t*)s.lines.p, n_lines,
                                    (int32_t*)s.tokens.p, (int64_t*)s.tok_off.p, (float*)s.scores.p, s.stream));
    s.launches += n_lines > 0 ? 3 : 1;
    RH_CUDA(cudaMemcpyAsync(token_offsets, s.tok_off.p, off_bytes, cudaMemcpyDeviceToHost, s.stream));
    if (n_lines > 0)
        RH_CUDA(cudaMemcpyAsync(scores, s.scores.p, (size_t)n_lines * sizeof(float), cudaMemcpyDeviceToHost, s.stream));
    if (int rc = sync_and_check(s)) return rc;
    const int64_t n_tok = token_offsets[n_lines];
    if (n_tok < 0 || n_tok > rows) return fail(RH_ERR_CUDA, "CTC collapse produced an impossible token count");
    if (n_tok > 0) {
        RH_CUDA(cudaMemcpyAsync(tokens, s.tokens.p, (size_t)n_tok * sizeof(int32_t), cudaMemcpyDeviceToHost, s.stream));
        RH_CUDA(cudaStreamSynchronize(s.stream));
    }
    return RH_OK;
}

// Rewrites the class table (scale, bias per class; padded classes (0, -inf)) on every device.
int upload_table(rh_ctx* ctx, rh_weight* w, const float* bias) {
    const int n_pad = w->g.n_chunks * rh::kBlockN;
    std::vector<float> ctab((size_t)w->g.n_chunks * rh::kCtabFloats);
    for (int j = 0; j < n_pad; ++j) {
        const int t = j / rh::kBlockN, r = j % rh::kBlockN;
        ctab[(size_t)t * rh::kCtabFloats + r] = j < w->n ? w->host_scales[j] : 0.0f;
        ctab[(size_t)t * rh::kCtabFloats + rh::kBlockN + r] = j < w->n ? (bias ? bias[j] : 0.0f) : -INFINITY;
    }
    for (auto& p : w->per) {
        Slot* slot = nullptr;
        for (auto& sp : ctx->slots)
            if (sp->device == p.device) slot = sp.get();
        if (!slot) return fail(RH_ERR_INVALID_ARG, "weight device is not in this context");
        RH_CUDA(cudaSetDevice(p.device));
        // ordered after every kernel already queued on the slot stream that reads the table
        RH_CUDA(cudaMemcpyAsync(p.ctab, ctab.data(), ctab.size() * sizeof(float), cudaMemcpyHostToDevice,
                                slot->stream));
        RH_CUDA(cudaStreamSynchronize(slot->stream));
    }
    return RH_OK;
}

// ----------------------------------------------------------- no-allocation entry point
// Some callers cannot allocate device memory at run time: a host that pre-reserves all GPU
// memory for itself, code that must not call cudaMalloc/cudaFree inside a latency-critical
// loop (both synchronise the device), or an embedder with its own allocator that forbids
// foreign allocations. rh_head_decode_device_noalloc serves them: its only scratch (the
// per-split partial (max, sum, argmax) rows that the class-range split writes and the merge
// kernel reads) lives in this fixed file-scope device array.
constexpr int64_t kNoAllocScratchEntries = 262144;  // float4 entries: 4 MiB per GPU
static __device__ __align__(256) float4 g_noalloc_scratch[kNoAllocScratchEntries];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[256] = {};  // device address of g_noalloc_scratch, per device ordinal

// Set-up, once per device, with that device current: the array's name is only a host-side
// stand-in, so the device address comes from cudaGetSymbolAddress.
int noalloc_scratch(int device, float4** out) {
    if (device < 0 || device >= 256) return fail(RH_ERR_UNSUPPORTED, "device ordinal above 255");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr)
            return fail(RH_ERR_CUDA, std::string("cudaGetSymbolAddress(g_noalloc_scratch): ") + cudaGetErrorString(e));
        g_noalloc_ptr[device] = ptr;
    }
    *out = static_cast<float4*>(g_noalloc_ptr[device]);
    return RH_OK;
}

// ------------------------------------------------------------- sharded batches
// Runs job(d, slot) for the shards d = 0..nd-1 (shard d on slot d, one host thread per device
// when nd > 1), then redoes every failed shard on a healthy device (results do not depend on
// the device); an invalid-argument failure is returned as it is. Host-side failure injection:
// RH_FAULT_DEVICE=<slot>[,<slot>...] makes those slots fail their shards.
template <class Job>
int run_shards(int nd, Job&& job) {
    const std::vector<int> faults = injected_fault_slots();
    std::vector<int> rc(nd, RH_OK);
    std::vector<std::string> msg(nd);
    auto run = [&](int d, int on_slot) {
        if (std::find(faults.begin(), faults.end(), on_slot) != faults.end()) {
            rc[d] = RH_ERR_DEVICE_FAULT;
            msg[d] = "injected failure on slot " + std::to_string(on_slot);
            return;
        }
        rc[d] = job(d, on_slot);
        if (rc[d]) msg[d] = g_err;
    };
    if (nd == 1) {
        run(0, 0);
    } else {
        std::vector<std::thread> th;
        for (int d = 0; d < nd; ++d) th.emplace_back(run, d, d);
        for (auto& t : th) t.join();
    }
    int healthy = -1;
    for (int d = 0; d < nd; ++d)
        if (rc[d] == RH_OK && std::find(faults.begin(), faults.end(), d) == faults.end()) {
            healthy = d;
            break;
        }
    for (int d = 0; d < nd; ++d) {
        if (rc[d] == RH_OK) continue;
        if (rc[d] == RH_ERR_INVALID_ARG) return fail(rc[d], msg[d]);
        if (healthy < 0) return fail(RH_ERR_DEVICE_FAULT, "every device shard failed; last: " + msg[d]);
        run(d, healthy);
        if (rc[d] != RH_OK) return fail(rc[d], msg[d]);
    }
    return RH_OK;
}

// The head on `nb` lines of the SVTR tail's [nb][k][t_len] output on one slot (host memory).
int kt_on_slot(rh_ctx* ctx, const rh_weight* w, int slot, const float* x, int64_t nb, int64_t t_len, int32_t* idx,
               float* prob) {
    const int64_t rows = nb * t_len;
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    const rh_weight::Per* pw = weight_on(w, s.device);
    if (!pw) return fail(RH_ERR_INVALID_ARG, "weight was not packed for this context's devices");
    const size_t x_bytes = (size_t)rows * (size_t)w->k * sizeof(float);
    RH_CUDA(s.a.ensure(x_bytes));
    RH_CUDA(s.idx.ensure((size_t)rows * sizeof(int32_t)));
    RH_CUDA(s.prob.ensure((size_t)rows * sizeof(float)));
    RH_CUDA(cudaMemcpyAsync(s.a.p, x, x_bytes, cudaMemcpyHostToDevice, s.stream));
    if (int rc = enqueue_head(ctx, w, s, *pw, (const float*)s.a.p, rows, (int32_t*)s.idx.p, (float*)s.prob.p, nullptr,
                              false, s.stream, t_len))
        return rc;
    RH_CUDA(cudaMemcpyAsync(idx, s.idx.p, (size_t)rows * sizeof(int32_t), cudaMemcpyDeviceToHost, s.stream));
    RH_CUDA(cudaMemcpyAsync(prob, s.prob.p, (size_t)rows * sizeof(float), cudaMemcpyDeviceToHost, s.stream));
    return sync_and_check(s);
}

// The head and the GPU collapse of `nb` padded lines (line b valid for valid_t[b] <= t_len
// timesteps) on one slot: tokens (room for the shard's valid rows), token_offsets [nb + 1]
// from 0 and scores [nb] in host memory.
int kt_ctc_on_slot(rh_ctx* ctx, const rh_weight* w, int slot, const float* x, int64_t nb, int64_t t_len,
                   const int64_t* valid_t, int32_t* tokens, int64_t* token_offsets, float* scores) {
    std::vector<int64_t> ranges(2 * (size_t)nb);  // line starts, then line ends (rows of the shard)
    int64_t total = 0;
    for (int64_t b = 0; b < nb; ++b) {
        ranges[b] = b * t_len;
        ranges[nb + b] = b * t_len + valid_t[b];
        total += valid_t[b];
    }
    token_offsets[0] = 0;
    if (total == 0) {  // every line empty: no tokens, score 0
        for (int64_t b = 0; b < nb; ++b) {
            token_offsets[b + 1] = 0;
            scores[b] = 0.0f;
        }
        return RH_OK;
    }
    const int64_t rows = nb * t_len;
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    const rh_weight::Per* pw = weight_on(w, s.device);
    if (!pw) return fail(RH_ERR_INVALID_ARG, "weight was not packed for this context's devices");
    const size_t x_bytes = (size_t)rows * (size_t)w->k * sizeof(float);
    RH_CUDA(s.a.ensure(x_bytes));
    RH_CUDA(s.idx.ensure((size_t)rows * sizeof(int32_t)));
    RH_CUDA(s.prob.ensure((size_t)rows * sizeof(float)));
    RH_CUDA(s.lines.ensure(ranges.size() * sizeof(int64_t)));
    RH_CUDA(s.tok_off.ensure((size_t)(nb + 1) * sizeof(int64_t)));
    RH_CUDA(s.tokens.ensure((size_t)total * sizeof(int32_t)));
    RH_CUDA(s.scores.ensure((size_t)nb * sizeof(float)));
    RH_CUDA(cudaMemcpyAsync(s.a.p, x, x_bytes, cudaMemcpyHostToDevice, s.stream));
    if (int rc = enqueue_head(ctx, w, s, *pw, (const float*)s.a.p, rows, (int32_t*)s.idx.p, (float*)s.prob.p, nullptr,
                              false, s.stream, t_len))
        return rc;
    RH_CUDA(cudaMemcpyAsync(s.lines.p, ranges.data(), ranges.size() * sizeof(int64_t), cudaMemcpyHostToDevice,
                            s.stream));
    const int64_t* d_begin = (const int64_t*)s.lines.p;
    RH_CUDA(rh::launch_ctc_collapse((const int32_t*)s.idx.p, (const float*)s.prob.p, d_begin, nb, (int32_t*)s.tokens.p,
                                    (int64_t*)s.tok_off.p, (float*)s.scores.p, s.stream, d_begin + nb));
    s.launches += 3;
    RH_CUDA(cudaMemcpyAsync(token_offsets, s.tok_off.p, (size_t)(nb + 1) * sizeof(int64_t), cudaMemcpyDeviceToHost,
                            s.stream));
    RH_CUDA(cudaMemcpyAsync(scores, s.scores.p, (size_t)nb * sizeof(float), cudaMemcpyDeviceToHost, s.stream));
    if (int rc = sync_and_check(s)) return rc;
    const int64_t n_tok = token_offsets[nb];
    if (n_tok < 0 || n_tok > total) return fail(RH_ERR_CUDA, "CTC collapse produced an impossible token count");
    if (n_tok > 0) {
        RH_CUDA(cudaMemcpyAsync(tokens, s.tokens.p, (size_t)n_tok * sizeof(int32_t), cudaMemcpyDeviceToHost, s.stream));
        RH_CUDA(cudaStreamSynchronize(s.stream));
    }
    return RH_OK;
}

// ------------------------------------------------------ recognition preprocessing
// Target staged span when choosing a line's chunk (24 KB of shared memory per block); lines
// that downscale so much that even one output column needs more than rh::kRecSpanMax input
// columns are rejected as unsupported.
constexpr double kRecSpanTarget = 2048.0;  // three f32 planes: 24 KB
constexpr uint32_t kRecMaxDim = 1u << 30;   // crop sides above this are rejected
constexpr uint32_t kRecMaxHeight = 1u << 20;  // target heights above this are rejected

// `v as u32` for f32 (saturating, NaN -> 0).
uint32_t f32_as_u32(float v) {
    if (!(v > 0.0f)) return 0;
    if (v >= 4294967296.0f) return UINT32_MAX;
    return (uint32_t)v;
}

// RecPreprocess::process's width rule (src/preprocess/rec.rs:62-75).
uint32_t rec_width(uint32_t w, uint32_t h, uint32_t target_h, uint32_t max_w) {
    const uint32_t hh = std::max<uint32_t>(h, 1), th = std::max<uint32_t>(target_h, 1);
    const uint32_t mw = std::max<uint32_t>(max_w, 32);
    const float aspect = (float)w / (float)hh;
    return std::min(std::max(f32_as_u32(std::ceil((float)th * aspect)), 32u), mw);
}

// Upper bound of the input columns that `chunk` consecutive output columns of a w -> out_w
// axis read: (chunk - 1) * ratio + 2 s + 2, plus 2 for f32 rounding of the window ends.
long long rec_span_bound(double ratio, double s, int chunk) {
    return (long long)std::ceil((chunk - 1) * ratio + 2.0 * s + 4.0);
}

struct RecBatch {
    std::vector<uint32_t> out_w;
    uint32_t out_h = 1, wmax = 0;
};

// Validates a batch (dimensions, crop byte ranges inside [0, rgb_len)) and computes its shape.
int rec_validate(const int64_t* offs, const uint32_t* widths, const uint32_t* heights, int64_t n, uint32_t target_h,
                 uint32_t max_w, int64_t rgb_len, RecBatch& b) {
    if (n < 0) return fail(RH_ERR_INVALID_ARG, "negative line count");
    if (n > 0 && (!widths || !heights)) return fail(RH_ERR_INVALID_ARG, "null crop sizes");
    b.out_h = std::max<uint32_t>(target_h, 1);
    if (b.out_h > kRecMaxHeight) return fail(RH_ERR_UNSUPPORTED, "target height above 2^20");
    b.out_w.resize((size_t)n);
    b.wmax = 0;
    for (int64_t l = 0; l < n; ++l) {
        const uint32_t w = widths[l], h = heights[l];
        if (w > kRecMaxDim || h > kRecMaxDim)
            return fail(RH_ERR_UNSUPPORTED, "crop " + std::to_string(l) + " has a side above 2^30 pixels");
        b.out_w[l] = rec_width(w, h, target_h, max_w);
        b.wmax = std::max(b.wmax, b.out_w[l]);
        if (w == 0 || h == 0) continue;
        if (offs) {
            const int64_t bytes = (int64_t)w * (int64_t)h * 3;
            if (offs[l] < 0 || offs[l] > rgb_len || bytes > rgb_len - offs[l])
                return fail(RH_ERR_INVALID_ARG, "crop " + std::to_string(l) + " (" + std::to_string(w) + " x " +
                                                    std::to_string(h) + " RGB8 at byte " + std::to_string(offs[l]) +
                                                    ") lies outside the pixel buffer of " + std::to_string(rgb_len) +
                                                    " bytes");
        }
        const double rx = (double)w / (double)b.out_w[l];
        if (rec_span_bound(rx, std::max(rx, 1.0), 1) > rh::kRecSpanMax)
            return fail(RH_ERR_UNSUPPORTED, "crop " + std::to_string(l) + " (" + std::to_string(w) + " x " +
                                                std::to_string(h) + ") shrinks by more than " +
                                                std::to_string(rh::kRecSpanMax / 2 - 2) +
                                                "x horizontally; split it or pre-scale it");
    }
    if ((uint64_t)b.wmax + b.out_h > 65535ull * rh::kRecThreads)
        return fail(RH_ERR_UNSUPPORTED, "resized width + target height above 16,776,960");
    return RH_OK;
}

// Line descriptors of lines [l0, l1) of a validated batch, crop bytes rebased by `base`;
// tables are laid out from 0. span_cap receives the largest staged span the lines need.
void rec_describe(const int64_t* offs, const uint32_t* widths, const uint32_t* heights, int64_t l0, int64_t l1,
                  const RecBatch& b, int64_t base, std::vector<rh::RecLine>& lines, long long& n_coords,
                  long long& n_wts, int& span_cap, int& meta_cap) {
    lines.resize((size_t)(l1 - l0));
    n_coords = 0;
    n_wts = 0;
    span_cap = 1;
    meta_cap = 0;
    for (int64_t l = l0; l < l1; ++l) {
        rh::RecLine& L = lines[l - l0];
        L = rh::RecLine{};
        L.w = (int)widths[l];
        L.h = (int)heights[l];
        L.out_w = (int)b.out_w[l];
        L.chunk = 1;
        if (L.w == 0 || L.h == 0) {
            L.w = 0;
            L.h = 0;
            continue;
        }
        L.src = offs[l] - base;
        const double rx = (double)L.w / L.out_w, sx = std::max(rx, 1.0);
        const double ry = (double)L.h / b.out_h, sy = std::max(ry, 1.0);
        // columns of a line that shrinks by at most 2x have at most ceil(2 s) <= 4 non-zero taps:
        // a zero-padded, 16-byte aligned slot of 4 (the window is trimmed in registers first)
        L.kx = sx <= 2.0 ? (int)std::ceil(2.0 * sx) : 0;
        L.stride_x = L.kx > 0 ? rh::kRecFastSlots : (int)std::ceil(2.0 * sx) + 3;
        L.stride_y = (int)std::ceil(2.0 * sy) + 3;
        // as many output columns per stage as keep the staged span within the target
        int chunk = L.out_w;
        if (rec_span_bound(rx, sx, chunk) > kRecSpanTarget)
            chunk = (int)std::min<double>(L.out_w,
                                          std::max(1.0, std::floor((kRecSpanTarget - 2.0 * sx - 4.0) / rx) + 1.0));
        L.chunk = chunk;
        span_cap = (int)std::max<long long>(span_cap, rec_span_bound(rx, sx, chunk));
        if (L.kx > 0 && chunk == L.out_w && L.out_w <= rh::kRecMetaMax) {
            meta_cap = std::max(meta_cap, L.out_w);
            span_cap = (int)std::max<long long>(span_cap, rec_span_bound(rx, sx, chunk) + 4);  // tap padding
        }
        L.coord = n_coords;
        n_wts = (n_wts + 3) & ~3LL;  // float4 loads of the column weights
        L.wts = n_wts;
        n_coords += (long long)L.out_w + b.out_h;
        n_wts += (long long)L.out_w * L.stride_x + (long long)b.out_h * L.stride_y;
    }
    // the staged windows share the block's shared memory with the span stage (227 KB per block)
    if ((3LL * span_cap + 3) / 4 * 16 + (long long)meta_cap * 20 > 200 * 1024) meta_cap = 0;
}

// Byte range [lo, hi) of the non-empty crops among lines [l0, l1) (lo == hi when none).
void rec_byte_range(const int64_t* offs, const uint32_t* widths, const uint32_t* heights, int64_t l0, int64_t l1,
                    int64_t& lo, int64_t& hi) {
    lo = INT64_MAX;
    hi = 0;
    for (int64_t l = l0; l < l1; ++l) {
        if (widths[l] == 0 || heights[l] == 0) continue;
        lo = std::min(lo, offs[l]);
        hi = std::max(hi, offs[l] + (int64_t)widths[l] * (int64_t)heights[l] * 3);
    }
    if (lo > hi) lo = hi = 0;
}

// Makes the slot's line/tap tables hold n lines, n_coords windows and n_wts weights, and orders
// `stream` after every kernel of the previous preprocessing call on this slot (whatever its
// stream), so that the tables are not overwritten while that call still reads them.
int rec_tables(Slot& s, cudaStream_t stream, int64_t n, long long n_coords, long long n_wts) {
    if (!s.pre_done) RH_CUDA(cudaEventCreateWithFlags(&s.pre_done, cudaEventDisableTiming));
    const size_t b_lines = (size_t)std::max<int64_t>(n, 1) * sizeof(rh::RecLine);
    const size_t b_coords = (size_t)std::max<long long>(n_coords, 1) * sizeof(int2);
    const size_t b_wts = (size_t)std::max<long long>(n_wts, 1) * sizeof(float);
    if (b_lines > s.pre_lines.cap || b_coords > s.pre_coords.cap || b_wts > s.pre_wts.cap)
        RH_CUDA(cudaEventSynchronize(s.pre_done));  // the old buffers are freed below
    RH_CUDA(cudaStreamWaitEvent(stream, s.pre_done, 0));
    RH_CUDA(s.pre_lines.ensure(b_lines));
    RH_CUDA(s.pre_coords.ensure(b_coords));
    RH_CUDA(s.pre_wts.ensure(b_wts));
    return RH_OK;
}

// Lines [l0, l1) of a host-memory batch on one device: crops up in pieces on the copy stream
// while the previous piece resizes, each piece's rows back to the host as soon as they are done.
int rec_host_on_slot(rh_ctx* ctx, int slot, const uint8_t* rgb, const int64_t* offs, const uint32_t* widths,
                     const uint32_t* heights, int64_t l0, int64_t l1, const RecBatch& b, float* out) {
    if (l1 <= l0) return RH_OK;
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    int64_t b0, b1;
    rec_byte_range(offs, widths, heights, l0, l1, b0, b1);
    std::vector<rh::RecLine> lines;
    long long n_coords, n_wts;
    int span_cap, meta_cap;
    rec_describe(offs, widths, heights, l0, l1, b, b0, lines, n_coords, n_wts, span_cap, meta_cap);
    const int64_t n = l1 - l0;
    const size_t line_floats = (size_t)3 * b.out_h * b.wmax;
    if (int rc = rec_tables(s, s.stream, n, n_coords, n_wts)) return rc;
    RH_CUDA(s.pre_rgb.ensure((size_t)std::max<int64_t>(b1 - b0, 1)));
    RH_CUDA(s.pre_out.ensure(std::max<size_t>((size_t)n * line_floats * sizeof(float), 4)));
    rh::RecParams p{};
    p.rgb = (const uint8_t*)s.pre_rgb.p;
    p.lines = (const rh::RecLine*)s.pre_lines.p;
    p.n_lines = n;
    p.out_h = (int)b.out_h;
    p.wmax = (int)b.wmax;
    p.span_cap = span_cap;
    p.meta_cap = meta_cap;
    p.coords = (int2*)s.pre_coords.p;
    p.wts = (float*)s.pre_wts.p;
    p.out = (float*)s.pre_out.p;
    p.inv = 1.0f / 127.5f;
    p.status = s.d_status;
    RH_CUDA(cudaMemcpyAsync(s.pre_lines.p, lines.data(), (size_t)n * sizeof(rh::RecLine), cudaMemcpyHostToDevice,
                            s.stream));
    RH_CUDA(rh::launch_rec_weights(p, s.stream));
    s.launches++;
    // pieces of about 32 MB of output
    const int64_t piece = std::max<int64_t>(1, (int64_t)((32u << 20) / std::max<size_t>(line_floats * 4, 1)));
    const int64_t max_grid_lines = std::max<int64_t>(1, 0x7fffffffLL / b.out_h);
    const int64_t step = std::min(piece, max_grid_lines);
    for (int64_t p0 = 0; p0 < n; p0 += step) {
        const int64_t pn = std::min(step, n - p0);
        int64_t c0, c1;
        rec_byte_range(offs, widths, heights, l0 + p0, l0 + p0 + pn, c0, c1);
        if (c1 > c0) {
            RH_CUDA(cudaMemcpyAsync((uint8_t*)s.pre_rgb.p + (c0 - b0), rgb + c0, (size_t)(c1 - c0),
                                    cudaMemcpyHostToDevice, s.copy_stream));
            RH_CUDA(cudaEventRecord(s.copied, s.copy_stream));
            RH_CUDA(cudaStreamWaitEvent(s.stream, s.copied, 0));
        }
        RH_CUDA(rh::launch_rec_resize(p, p0, pn, s.stream));
        s.launches++;
        RH_CUDA(cudaMemcpyAsync(out + (size_t)(l0 + p0) * line_floats, (float*)s.pre_out.p + (size_t)p0 * line_floats,
                                (size_t)pn * line_floats * sizeof(float), cudaMemcpyDeviceToHost, s.stream));
    }
    RH_CUDA(cudaEventRecord(s.pre_done, s.stream));
    return sync_and_check(s);
}

}  // namespace

extern "C" {

int rh_version(void) { return 100; }

const char* rh_last_error(void) { return g_err.c_str(); }

int rh_device_count(int* count) {
    if (!count) return fail(RH_ERR_INVALID_ARG, "count is null");
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    if (e != cudaSuccess) c = 0;
    *count = c;
    return RH_OK;
}

int rh_ctx_create(const int* devices, int n_devices, rh_ctx** out) {
    if (!out) return fail(RH_ERR_INVALID_ARG, "out is null");
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
        return fail(RH_ERR_NO_DEVICE, "no CUDA device is visible; this library has no CPU path");
    std::vector<int> devs;
    if (!devices || n_devices <= 0)
        devs.push_back(0);
    else
        devs.assign(devices, devices + n_devices);
    auto ctx = std::make_unique<rh_ctx>();
    if (const char* t = std::getenv("RH_TIMEOUT_MS")) ctx->timeout_ns = (unsigned long long)std::atoll(t) * 1000000ull;
    for (int d : devs) {
        if (d < 0 || d >= count) return fail(RH_ERR_INVALID_ARG, "device index out of range: " + std::to_string(d));
        for (const auto& s : ctx->slots)
            if (s->device == d) return fail(RH_ERR_INVALID_ARG, "device listed twice: " + std::to_string(d));
        cudaDeviceProp prop;
        RH_CUDA(cudaGetDeviceProperties(&prop, d));
        if (prop.major != 10 || prop.minor != 0)
            return fail(RH_ERR_UNSUPPORTED, std::string("device ") + std::to_string(d) + " (" + prop.name + ", sm_" +
                                                std::to_string(prop.major) + std::to_string(prop.minor) +
                                                ") is not sm_100; the kernels are built for sm_100a only");
        auto s = std::make_unique<Slot>();
        s->device = d;
        s->sms = prop.multiProcessorCount;
        RH_CUDA(cudaSetDevice(d));
        RH_CUDA(rh::head_kernel_setup());
        RH_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
        RH_CUDA(cudaStreamCreateWithFlags(&s->copy_stream, cudaStreamNonBlocking));
        RH_CUDA(cudaEventCreateWithFlags(&s->copied, cudaEventDisableTiming));
        RH_CUDA(cudaMalloc(&s->d_status, 2 * sizeof(int)));
        RH_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&s->h_status), 2 * sizeof(int), cudaHostAllocDefault));
        RH_CUDA(cudaMemsetAsync(s->d_status, 0, 2 * sizeof(int), s->stream));
        RH_CUDA(cudaStreamSynchronize(s->stream));
        ctx->slots.push_back(std::move(s));
    }
    *out = ctx.release();
    return RH_OK;
}

void rh_ctx_destroy(rh_ctx* ctx) {
    delete ctx;  // each Slot waits for its streams and frees its buffers
}

int rh_ctx_num_devices(const rh_ctx* ctx) { return ctx ? (int)ctx->slots.size() : 0; }

int rh_ctx_set_timeout_ms(rh_ctx* ctx, int timeout_ms) {
    if (int rc = check_ctx(ctx)) return rc;
    if (timeout_ms <= 0) return fail(RH_ERR_INVALID_ARG, "timeout must be positive");
    ctx->timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
    return RH_OK;
}

namespace {
int pack_weight(rh_ctx* ctx, const float* w_nk, int64_t n, int64_t k, const float* bias, int64_t bias_len, bool f32,
                bool compact, rh_weight** out) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!out || !w_nk) return fail(RH_ERR_INVALID_ARG, "null weight or output pointer");
    *out = nullptr;
    if (n < 1 || k < 1) return fail(RH_ERR_INVALID_ARG, "weight must be [n>=1][k>=1]");
    if (k > rh::kPadK)
        return fail(RH_ERR_UNSUPPORTED, "K = " + std::to_string(k) + " exceeds the supported maximum of 128");
    if (n > (int64_t)1 << 24) return fail(RH_ERR_UNSUPPORTED, "n too large");
    if (bias && bias_len != n)
        return fail(RH_ERR_INVALID_ARG,
                    "bias has " + std::to_string(bias_len) + " elements but n is " + std::to_string(n));
    auto w = std::make_unique<rh_weight>();
    w->n = n;
    w->k = k;
    w->f32 = f32;
    w->compact = compact && !f32;
    w->g = geometry(n, k);
    const int n_pad = w->g.n_chunks * rh::kBlockN;
    for (auto& sp : ctx->slots) {
        Slot& s = *sp;
        std::lock_guard<std::mutex> lock(s.mu);
        RH_CUDA(cudaSetDevice(s.device));
        rh_weight::Per p;
        p.device = s.device;
        RH_CUDA(cudaMalloc(&p.tiles, (size_t)w->g.n_chunks * w->tile_bytes()));
        RH_CUDA(cudaMalloc(&p.ctab, (size_t)w->g.n_chunks * rh::kCtabFloats * sizeof(float)));
        w->per.push_back(p);
        DevBuf tw, tb;  // temporaries, freed on every path
        RH_CUDA(tw.ensure((size_t)n * (size_t)k * sizeof(float)));
        float* d_w = static_cast<float*>(tw.p);
        float* d_b = nullptr;
        // Stream-ordered copies: a plain cudaMemcpy from pageable memory may return before its
        // DMA lands, and the pack kernel runs on a non-blocking stream.
        RH_CUDA(cudaMemcpyAsync(d_w, w_nk, (size_t)n * (size_t)k * sizeof(float), cudaMemcpyHostToDevice, s.stream));
        if (bias) {
            RH_CUDA(tb.ensure((size_t)n * sizeof(float)));
            d_b = static_cast<float*>(tb.p);
            RH_CUDA(cudaMemcpyAsync(d_b, bias, (size_t)n * sizeof(float), cudaMemcpyHostToDevice, s.stream));
        }
        rh::PackParams pp{};
        pp.w = d_w;
        pp.bias = d_b;
        pp.n = (int)n;
        pp.k = (int)k;
        pp.n_pad = n_pad;
        pp.merged_tail = w->g.merged;
        pp.tail_step = w->g.tail_step;
        pp.f32 = f32 ? 1 : 0;
        pp.compact = w->compact ? 1 : 0;
        pp.btiles = p.tiles;
        pp.ctab = p.ctab;
        RH_CUDA(rh::launch_pack(pp, s.stream));
        s.launches++;
        RH_CUDA(cudaStreamSynchronize(s.stream));
        if (w->host_scales.empty()) {  // the per-class scales, read back from the class table
            std::vector<float> ctab((size_t)w->g.n_chunks * rh::kCtabFloats);
            RH_CUDA(cudaMemcpyAsync(ctab.data(), p.ctab, ctab.size() * sizeof(float), cudaMemcpyDeviceToHost,
                                    s.stream));
            RH_CUDA(cudaStreamSynchronize(s.stream));
            w->host_scales.resize((size_t)n);
            for (int64_t j = 0; j < n; ++j)
                w->host_scales[(size_t)j] = ctab[(size_t)(j / rh::kBlockN) * rh::kCtabFloats + (size_t)(j % rh::kBlockN)];
        }
    }
    *out = w.release();
    return RH_OK;
}
}  // namespace

int rh_weight_pack(rh_ctx* ctx, const float* w_nk, int64_t n, int64_t k, const float* bias, int64_t bias_len,
                   rh_weight** out) {
    return pack_weight(ctx, w_nk, n, k, bias, bias_len, false, false, out);
}

int rh_weight_pack_compact(rh_ctx* ctx, const float* w_nk, int64_t n, int64_t k, const float* bias, int64_t bias_len,
                           rh_weight** out) {
    return pack_weight(ctx, w_nk, n, k, bias, bias_len, false, true, out);
}

int rh_weight_pack_f32(rh_ctx* ctx, const float* w_nk, int64_t n, int64_t k, const float* bias, int64_t bias_len,
                       rh_weight** out) {
    return pack_weight(ctx, w_nk, n, k, bias, bias_len, true, false, out);
}

int rh_weight_set_bias(rh_ctx* ctx, rh_weight* w, const float* bias, int64_t bias_len) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (bias && bias_len != w->n)
        return fail(RH_ERR_INVALID_ARG,
                    "bias has " + std::to_string(bias_len) + " elements but n is " + std::to_string(w->n));
    for (auto& s : ctx->slots) s->mu.lock();
    int rc = upload_table(ctx, w, bias);
    for (auto& s : ctx->slots) s->mu.unlock();
    return rc;
}

int rh_weight_export(rh_ctx* ctx, const rh_weight* w, int8_t* q, float* scales) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w || w->per.empty()) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (w->f32) return fail(RH_ERR_INVALID_ARG, "an FP32 weight has no int8 data");
    const auto& p = w->per[0];
    RH_CUDA(cudaSetDevice(p.device));
    RH_CUDA(cudaDeviceSynchronize());
    if (q) {  // QuantizedWeight::data read back from the tiles (fp16 image, or int8 stored as q + 128)
        std::vector<uint8_t> img((size_t)w->g.n_chunks * w->tile_bytes());
        RH_CUDA(cudaMemcpy(img.data(), p.tiles, img.size(), cudaMemcpyDeviceToHost));
        for (int64_t j = 0; j < w->n; ++j) {
            const uint8_t* tile = img.data() + (size_t)(j / rh::kBlockN) * w->tile_bytes();
            const int r = (int)(j % rh::kBlockN);
            for (int64_t s = 0; s < w->k; ++s) {
                int v;
                if (w->compact) {
                    v = (int)tile[rh::image8_offset(r, (int)s)] - 128;
                } else {  // integer-valued fp16 (|q| <= 127): sign, exponent and 10-bit fraction
                    const uint32_t off = (uint32_t)(s >> 6) * 16384u + (uint32_t)r * 128u +
                                         (uint32_t)((((s & 63) >> 3) ^ (r & 7)) << 4) + (uint32_t)(s & 7) * 2u;
                    const uint16_t h = (uint16_t)(tile[off] | (tile[off + 1] << 8));
                    const int e = (h >> 10) & 31;
                    const int mag = e == 0 ? 0 : (int)(((h & 1023) | 1024) >> (25 - e));
                    v = (h & 0x8000) ? -mag : mag;
                }
                q[(size_t)j * (size_t)w->k + (size_t)s] = (int8_t)v;
            }
        }
    }
    if (scales) std::memcpy(scales, w->host_scales.data(), (size_t)w->n * sizeof(float));
    return RH_OK;
}

int rh_weight_export_image(rh_ctx* ctx, const rh_weight* w, uint8_t* tiles, float* table) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w || w->per.empty()) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (w->f32) return fail(RH_ERR_INVALID_ARG, "the image of an FP32 weight is not exported");
    const auto& p = w->per[0];
    RH_CUDA(cudaSetDevice(p.device));
    RH_CUDA(cudaDeviceSynchronize());
    if (tiles) RH_CUDA(cudaMemcpy(tiles, p.tiles, (size_t)w->g.n_chunks * w->tile_bytes(), cudaMemcpyDeviceToHost));
    if (table)
        RH_CUDA(cudaMemcpy(table, p.ctab, (size_t)w->g.n_chunks * rh::kCtabFloats * sizeof(float),
                           cudaMemcpyDeviceToHost));
    return RH_OK;
}

int rh_weight_dims(const rh_weight* w, int64_t* n, int64_t* k) {
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (n) *n = w->n;
    if (k) *k = w->k;
    return RH_OK;
}

int64_t rh_weight_tile_bytes(const rh_weight* w) { return w ? (int64_t)w->tile_bytes() : 0; }

int64_t rh_weight_device_bytes(const rh_weight* w) {
    if (!w) return 0;
    return (int64_t)w->g.n_chunks * ((int64_t)w->tile_bytes() + rh::kCtabFloats * (int64_t)sizeof(float));
}

void rh_weight_free(rh_weight* w) {
    delete w;  // frees every device copy
}

int rh_matmul_quantized_b(rh_ctx* ctx, const rh_weight* w, const float* a, int64_t rows, int64_t k, float* out) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (w->f32) return fail(RH_ERR_INVALID_ARG, "weight was packed FP32: use rh_matmul_transposed_b");
    if (k != w->k)
        return fail(RH_ERR_INVALID_ARG,
                    "Inner dimensions must match: " + std::to_string(k) + " != " + std::to_string(w->k));
    if (rows < 0) return fail(RH_ERR_INVALID_ARG, "negative row count");
    if (rows == 0) return RH_OK;
    if (!a || !out) return fail(RH_ERR_INVALID_ARG, "null input or output");
    return run_host_on_slot(ctx, w, 0, a, rows, nullptr, nullptr, out);
}

int rh_matmul_transposed_b(rh_ctx* ctx, const rh_weight* w, const float* a, int64_t rows, int64_t k, float* out) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (!w->f32) return fail(RH_ERR_INVALID_ARG, "weight was packed INT8: use rh_matmul_quantized_b");
    if (k != w->k)
        return fail(RH_ERR_INVALID_ARG,
                    "Inner dimensions must match: " + std::to_string(k) + " != " + std::to_string(w->k));
    if (rows < 0) return fail(RH_ERR_INVALID_ARG, "negative row count");
    if (rows == 0) return RH_OK;
    if (!a || !out) return fail(RH_ERR_INVALID_ARG, "null input or output");
    return run_host_on_slot(ctx, w, 0, a, rows, nullptr, nullptr, out);
}

int rh_head_decode(rh_ctx* ctx, const rh_weight* w, const float* a, int64_t rows, int64_t k, int32_t* idx,
                   float* prob) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (k != w->k)
        return fail(RH_ERR_INVALID_ARG,
                    "Inner dimensions must match: " + std::to_string(k) + " != " + std::to_string(w->k));
    if (rows < 0) return fail(RH_ERR_INVALID_ARG, "negative row count");
    if (rows == 0) return RH_OK;
    if (!a || !idx || !prob) return fail(RH_ERR_INVALID_ARG, "null input or output");
    return run_host_on_slot(ctx, w, 0, a, rows, idx, prob, nullptr);
}

int rh_head_decode_lines(rh_ctx* ctx, const rh_weight* w, const float* a, const int64_t* line_offsets,
                         int64_t n_lines, int64_t k, int32_t* idx, float* prob) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (k != w->k)
        return fail(RH_ERR_INVALID_ARG,
                    "Inner dimensions must match: " + std::to_string(k) + " != " + std::to_string(w->k));
    if (n_lines < 0 || (n_lines > 0 && !line_offsets)) return fail(RH_ERR_INVALID_ARG, "bad line offsets");
    if (n_lines == 0) return RH_OK;
    if (line_offsets[0] < 0) return fail(RH_ERR_INVALID_ARG, "line offsets must start at >= 0");
    for (int64_t l = 0; l < n_lines; ++l)
        if (line_offsets[l + 1] < line_offsets[l]) return fail(RH_ERR_INVALID_ARG, "line offsets must not decrease");
    const int64_t r0 = line_offsets[0], total = line_offsets[n_lines] - r0;
    if (total == 0) return RH_OK;
    if (!a || !idx || !prob) return fail(RH_ERR_INVALID_ARG, "null input or output");

    // Contiguous line shards with balanced timestep counts, one per device.
    const int nd = (int)ctx->slots.size();
    std::vector<int64_t> cut(nd + 1, r0);
    cut[nd] = r0 + total;
    int64_t l = 0;
    for (int d = 1; d < nd; ++d) {
        const int64_t target = r0 + (total * d) / nd;
        while (l < n_lines && line_offsets[l] < target) ++l;
        cut[d] = std::max(cut[d - 1], std::min(line_offsets[l], r0 + total));
    }
    return run_shards(nd, [&](int d, int slot) -> int {
        const int64_t rows = cut[d + 1] - cut[d];
        if (rows <= 0) return RH_OK;
        return run_host_on_slot(ctx, w, slot, a + (size_t)(cut[d] - r0) * (size_t)k, rows, idx + (cut[d] - r0),
                                prob + (cut[d] - r0), nullptr);
    });
}

int rh_head_decode_kt_device(rh_ctx* ctx, const rh_weight* w, int slot, const float* d_x, int64_t batch,
                             int64_t t_len, int32_t* d_idx, float* d_prob, void* stream) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (slot < 0 || slot >= (int)ctx->slots.size()) return fail(RH_ERR_INVALID_ARG, "slot out of range");
    if (batch < 0 || t_len < 0) return fail(RH_ERR_INVALID_ARG, "negative batch or sequence length");
    if (batch == 0 || t_len == 0) return RH_OK;
    if (!d_x || !d_idx || !d_prob) return fail(RH_ERR_INVALID_ARG, "null device pointer");
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    const rh_weight::Per* pw = weight_on(w, s.device);
    if (!pw) return fail(RH_ERR_INVALID_ARG, "weight was not packed for this device");
    return enqueue_head(ctx, w, s, *pw, d_x, batch * t_len, d_idx, d_prob, nullptr, false, (cudaStream_t)stream,
                        t_len);
}

int rh_head_decode_kt(rh_ctx* ctx, const rh_weight* w, const float* x, int64_t batch, int64_t k, int64_t t_len,
                      int32_t* idx, float* prob) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (k != w->k)
        return fail(RH_ERR_INVALID_ARG,
                    "Inner dimensions must match: " + std::to_string(k) + " != " + std::to_string(w->k));
    if (batch < 0 || t_len < 0) return fail(RH_ERR_INVALID_ARG, "negative batch or sequence length");
    const int64_t rows = batch * t_len;
    if (rows == 0) return RH_OK;
    if (!x || !idx || !prob) return fail(RH_ERR_INVALID_ARG, "null input or output");
    // contiguous line shards of equal size (every line has t_len timesteps), one per device
    const int nd = (int)ctx->slots.size();
    return run_shards(nd, [&](int d, int slot) -> int {
        const int64_t b0 = batch * d / nd, b1 = batch * (d + 1) / nd;
        if (b1 <= b0) return RH_OK;
        return kt_on_slot(ctx, w, slot, x + (size_t)b0 * (size_t)k * (size_t)t_len, b1 - b0, t_len,
                          idx + b0 * t_len, prob + b0 * t_len);
    });
}

int rh_head_decode_kt_ctc(rh_ctx* ctx, const rh_weight* w, const float* x, int64_t batch, int64_t k, int64_t t_len,
                          const int64_t* valid_t, int32_t* tokens, int64_t* token_offsets, float* scores) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (k != w->k)
        return fail(RH_ERR_INVALID_ARG,
                    "Inner dimensions must match: " + std::to_string(k) + " != " + std::to_string(w->k));
    if (batch < 0 || t_len < 0) return fail(RH_ERR_INVALID_ARG, "negative batch or sequence length");
    if (!token_offsets) return fail(RH_ERR_INVALID_ARG, "null token offsets");
    token_offsets[0] = 0;
    if (batch == 0) return RH_OK;
    if (!valid_t || !scores) return fail(RH_ERR_INVALID_ARG, "null valid lengths or scores");
    std::vector<int64_t> vstart((size_t)batch + 1, 0);  // valid rows before each line
    for (int64_t b = 0; b < batch; ++b) {
        if (valid_t[b] < 0 || valid_t[b] > t_len)
            return fail(RH_ERR_INVALID_ARG, "valid length " + std::to_string(valid_t[b]) + " of line " +
                                                std::to_string(b) + " is outside [0, " + std::to_string(t_len) + "]");
        vstart[b + 1] = vstart[b] + valid_t[b];
    }
    if (vstart[batch] > 0 && (!x || !tokens)) return fail(RH_ERR_INVALID_ARG, "null input or tokens");
    // contiguous line shards of equal size, one per device; shard d writes its tokens from its
    // first valid row's position and the shards are packed back to back at the end
    const int nd = (int)ctx->slots.size();
    std::vector<std::vector<int64_t>> local_off(nd);
    int rc = run_shards(nd, [&](int d, int slot) -> int {
        const int64_t b0 = batch * d / nd, b1 = batch * (d + 1) / nd;
        local_off[d].assign((size_t)(b1 - b0) + 1, 0);
        if (b1 <= b0) return RH_OK;
        return kt_ctc_on_slot(ctx, w, slot, x + (size_t)b0 * (size_t)k * (size_t)t_len, b1 - b0, t_len, valid_t + b0,
                              tokens + vstart[b0], local_off[d].data(), scores + b0);
    });
    if (rc) return rc;
    int64_t wpos = 0;
    for (int d = 0; d < nd; ++d) {
        const int64_t b0 = batch * d / nd, b1 = batch * (d + 1) / nd;
        if (b1 <= b0) continue;
        const int64_t n_tok = local_off[d][b1 - b0];
        if (n_tok > 0 && vstart[b0] != wpos) std::memmove(tokens + wpos, tokens + vstart[b0], (size_t)n_tok * sizeof(int32_t));
        for (int64_t b = b0; b < b1; ++b) token_offsets[b] = wpos + local_off[d][b - b0];
        wpos += n_tok;
    }
    token_offsets[batch] = wpos;
    return RH_OK;
}

int rh_head_decode_device(rh_ctx* ctx, const rh_weight* w, int slot, const float* d_a, int64_t rows, int32_t* d_idx,
                          float* d_prob, void* stream) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (slot < 0 || slot >= (int)ctx->slots.size()) return fail(RH_ERR_INVALID_ARG, "slot out of range");
    if (rows < 0) return fail(RH_ERR_INVALID_ARG, "negative row count");
    if (rows == 0) return RH_OK;
    if (!d_a || !d_idx || !d_prob) return fail(RH_ERR_INVALID_ARG, "null device pointer");
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    const rh_weight::Per* pw = weight_on(w, s.device);
    if (!pw) return fail(RH_ERR_INVALID_ARG, "weight was not packed for this device");
    return enqueue_head(ctx, w, s, *pw, d_a, rows, d_idx, d_prob, nullptr, false, (cudaStream_t)stream);
}

int rh_matmul_quantized_b_device(rh_ctx* ctx, const rh_weight* w, int slot, const float* d_a, int64_t rows,
                                 float* d_out, void* stream) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (slot < 0 || slot >= (int)ctx->slots.size()) return fail(RH_ERR_INVALID_ARG, "slot out of range");
    if (rows < 0) return fail(RH_ERR_INVALID_ARG, "negative row count");
    if (rows == 0) return RH_OK;
    if (!d_a || !d_out) return fail(RH_ERR_INVALID_ARG, "null device pointer");
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    const rh_weight::Per* pw = weight_on(w, s.device);
    if (!pw) return fail(RH_ERR_INVALID_ARG, "weight was not packed for this device");
    return enqueue_head(ctx, w, s, *pw, d_a, rows, nullptr, nullptr, d_out, true, (cudaStream_t)stream);
}

int rh_sync(rh_ctx* ctx, int slot) {
    if (int rc = check_ctx(ctx)) return rc;
    int first = slot < 0 ? 0 : slot, last = slot < 0 ? (int)ctx->slots.size() - 1 : slot;
    if (first < 0 || last >= (int)ctx->slots.size()) return fail(RH_ERR_INVALID_ARG, "slot out of range");
    int result = RH_OK;
    for (int i = first; i <= last; ++i) {
        Slot& s = *ctx->slots[i];
        std::lock_guard<std::mutex> lock(s.mu);
        RH_CUDA(cudaSetDevice(s.device));
        RH_CUDA(cudaDeviceSynchronize());
        int rc = read_status(s);
        if (rc && !result) result = rc;
    }
    return result;
}

int64_t rh_launch_count(const rh_ctx* ctx, int slot) {
    if (!ctx || slot < 0 || slot >= (int)ctx->slots.size()) return -1;
    return ctx->slots[slot]->launches;
}

int64_t rh_ctc_collapse(const int32_t* idx, const float* prob, const int64_t* line_offsets, int64_t n_lines,
                        int32_t* tokens, int64_t* token_offsets, float* scores) {
    if (n_lines < 0 || !line_offsets || !token_offsets || (n_lines > 0 && !scores)) {
        g_err = "rh_ctc_collapse: bad arguments";
        return -1;
    }
    for (int64_t l = 0; l < n_lines; ++l)
        if (line_offsets[l + 1] < line_offsets[l] || line_offsets[l] < 0) {
            g_err = "rh_ctc_collapse: line offsets must not decrease";
            return -1;
        }
    if (n_lines > 0 && line_offsets[n_lines] > line_offsets[0] && (!idx || !prob || !tokens)) {
        g_err = "rh_ctc_collapse: null idx/prob/tokens";
        return -1;
    }
    int64_t w = 0;
    for (int64_t l = 0; l < n_lines; ++l) {
        token_offsets[l] = w;
        int32_t last = 0;
        float sum = 0.0f;
        int64_t count = 0;
        for (int64_t t = line_offsets[l]; t < line_offsets[l + 1]; ++t) {
            const int32_t c = idx[t];
            if (c != 0 && c != last) {
                tokens[w++] = c;
                sum += prob[t];
                ++count;
            }
            last = c;
        }
        scores[l] = count == 0 ? 0.0f : sum / (float)count;
    }
    token_offsets[n_lines] = w;
    return w;
}


int rh_ctc_collapse_device(rh_ctx* ctx, int slot, const int32_t* d_idx, const float* d_prob,
                           const int64_t* d_line_offsets, int64_t n_lines, int32_t* d_tokens, int64_t* d_token_offsets,
                           float* d_scores, void* stream) {
    if (int rc = check_ctx(ctx)) return rc;
    if (slot < 0 || slot >= (int)ctx->slots.size()) return fail(RH_ERR_INVALID_ARG, "slot out of range");
    if (n_lines < 0) return fail(RH_ERR_INVALID_ARG, "negative line count");
    if (!d_token_offsets) return fail(RH_ERR_INVALID_ARG, "null device pointer");
    if (n_lines > 0 && (!d_idx || !d_prob || !d_line_offsets || !d_tokens || !d_scores))
        return fail(RH_ERR_INVALID_ARG, "null device pointer");
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    RH_CUDA(rh::launch_ctc_collapse(d_idx, d_prob, d_line_offsets, n_lines, d_tokens, d_token_offsets, d_scores,
                                    (cudaStream_t)stream));
    s.launches += n_lines > 0 ? 3 : 1;
    return RH_OK;
}

int rh_head_decode_ctc(rh_ctx* ctx, const rh_weight* w, const float* a, const int64_t* line_offsets, int64_t n_lines,
                       int64_t k, int32_t* tokens, int64_t* token_offsets, float* scores) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (k != w->k)
        return fail(RH_ERR_INVALID_ARG,
                    "Inner dimensions must match: " + std::to_string(k) + " != " + std::to_string(w->k));
    if (n_lines < 0 || !line_offsets || !token_offsets) return fail(RH_ERR_INVALID_ARG, "bad line offsets");
    if (line_offsets[0] < 0) return fail(RH_ERR_INVALID_ARG, "line offsets must start at >= 0");
    for (int64_t l = 0; l < n_lines; ++l)
        if (line_offsets[l + 1] < line_offsets[l]) return fail(RH_ERR_INVALID_ARG, "line offsets must not decrease");
    token_offsets[0] = 0;
    if (n_lines == 0) return RH_OK;
    const int64_t r0 = line_offsets[0], total = line_offsets[n_lines] - r0;
    if (!scores || (total > 0 && (!a || !tokens))) return fail(RH_ERR_INVALID_ARG, "null input or output");

    // Contiguous line shards with balanced timestep counts, one per device (as in
    // rh_head_decode_lines); shard d writes its tokens at its own row range of `tokens`, and
    // the shards are packed back to back once all have finished.
    const int nd = (int)ctx->slots.size();
    std::vector<int64_t> lcut(nd + 1, 0);
    lcut[nd] = n_lines;
    for (int d = 1; d < nd; ++d) {
        const int64_t target = r0 + (total * d) / nd;
        int64_t l = lcut[d - 1];
        while (l < n_lines && line_offsets[l] < target) ++l;
        lcut[d] = l;
    }
    std::vector<std::vector<int64_t>> local_off(nd);
    int rc = run_shards(nd, [&](int d, int slot) -> int {
        const int64_t l0 = lcut[d], l1 = lcut[d + 1];
        local_off[d].assign((size_t)(l1 - l0) + 1, 0);
        if (l1 <= l0) return RH_OK;
        std::vector<int64_t> lo(l1 - l0 + 1);
        for (int64_t l = l0; l <= l1; ++l) lo[l - l0] = line_offsets[l] - line_offsets[l0];
        return run_ctc_on_slot(ctx, w, slot, a + (size_t)(line_offsets[l0] - r0) * (size_t)k, lo.data(), l1 - l0,
                               tokens + (line_offsets[l0] - r0), local_off[d].data(), scores + l0);
    });
    if (rc) return rc;
    // pack the shards' tokens back to back (each shard's tokens sit at the start of its rows)
    int64_t wpos = 0;
    for (int d = 0; d < nd; ++d) {
        const int64_t l0 = lcut[d], l1 = lcut[d + 1];
        if (l1 <= l0) continue;
        const int64_t n_tok = local_off[d][l1 - l0];
        const int64_t src = line_offsets[l0] - r0;
        if (n_tok > 0 && src != wpos) std::memmove(tokens + wpos, tokens + src, (size_t)n_tok * sizeof(int32_t));
        for (int64_t l = l0; l < l1; ++l) token_offsets[l] = wpos + local_off[d][l - l0];
        wpos += n_tok;
    }
    token_offsets[n_lines] = wpos;
    return RH_OK;
}

int rh_head_decode_device_noalloc(rh_ctx* ctx, const rh_weight* w, int slot, const float* d_a, int64_t rows,
                                  int32_t* d_idx, float* d_prob, void* stream) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!w) return fail(RH_ERR_INVALID_ARG, "null weight");
    if (slot < 0 || slot >= (int)ctx->slots.size()) return fail(RH_ERR_INVALID_ARG, "slot out of range");
    if (rows < 0) return fail(RH_ERR_INVALID_ARG, "negative row count");
    if (rows > kNoAllocScratchEntries)
        return fail(RH_ERR_INVALID_ARG, "rh_head_decode_device_noalloc: " + std::to_string(rows) +
                                            " rows exceed its static limit of " +
                                            std::to_string(kNoAllocScratchEntries) +
                                            " timestep rows per call; split the batch or use rh_head_decode_device");
    if (rows == 0) return RH_OK;
    if (!d_a || !d_idx || !d_prob) return fail(RH_ERR_INVALID_ARG, "null device pointer");
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    const rh_weight::Per* pw = weight_on(w, s.device);
    if (!pw) return fail(RH_ERR_INVALID_ARG, "weight was not packed for this device");
    float4* scratch = nullptr;
    if (int rc = noalloc_scratch(s.device, &scratch)) return rc;

    int grid;
    rh::HeadParams p = head_params(ctx, w, s, *pw, d_a, rows, 0, d_idx, d_prob, nullptr, grid);
    // Partial entries: splits x the rows of the split row blocks, which are fewer than one
    // wave (148 x 128 rows); the planner keeps splits x those blocks near one wave, so the
    // plan fits the array at any call size. The check only guards that.
    const int64_t entries = (int64_t)p.n_splits * split_rows(p);
    if (entries > kNoAllocScratchEntries)
        return fail(RH_ERR_UNSUPPORTED, "rh_head_decode_device_noalloc: the work plan needs " + std::to_string(entries) +
                                            " partial entries, more than its static array holds");
    p.partial = split_rows(p) > 0 ? scratch : nullptr;
    return launch_head_and_merge(s, p, false, grid, (cudaStream_t)stream);
}

// ------------------------------------------------------ recognition preprocessing

uint32_t rh_rec_resized_width(uint32_t orig_w, uint32_t orig_h, uint32_t target_h, uint32_t max_w) {
    return rec_width(orig_w, orig_h, target_h, max_w);
}

int rh_rec_batch_shape(const uint32_t* widths, const uint32_t* heights, int64_t n_lines, uint32_t target_h,
                       uint32_t max_w, uint32_t* out_widths, uint32_t* out_h, uint32_t* out_wmax) {
    RecBatch b;
    if (int rc = rec_validate(nullptr, widths, heights, n_lines, target_h, max_w, 0, b)) return rc;
    if (out_widths && n_lines > 0) std::memcpy(out_widths, b.out_w.data(), (size_t)n_lines * sizeof(uint32_t));
    if (out_h) *out_h = b.out_h;
    if (out_wmax) *out_wmax = b.wmax;
    return RH_OK;
}

int rh_rec_preprocess(rh_ctx* ctx, const uint8_t* rgb, int64_t rgb_len, const int64_t* rgb_offsets,
                      const uint32_t* widths, const uint32_t* heights, int64_t n_lines, uint32_t target_h,
                      uint32_t max_w, float* out, int64_t out_len, uint32_t* out_widths, uint32_t* out_wmax) {
    if (int rc = check_ctx(ctx)) return rc;
    if (rgb_len < 0) return fail(RH_ERR_INVALID_ARG, "negative pixel buffer length");
    if (n_lines > 0 && !rgb_offsets) return fail(RH_ERR_INVALID_ARG, "null crop offsets");
    RecBatch b;
    if (int rc = rec_validate(rgb_offsets, widths, heights, n_lines, target_h, max_w, rgb_len, b)) return rc;
    if (out_widths && n_lines > 0) std::memcpy(out_widths, b.out_w.data(), (size_t)n_lines * sizeof(uint32_t));
    if (out_wmax) *out_wmax = b.wmax;
    if (n_lines == 0) return RH_OK;
    const long double need = (long double)n_lines * 3.0L * b.out_h * b.wmax;
    if (!out || (long double)out_len < need)
        return fail(RH_ERR_INVALID_ARG, "output holds " + std::to_string(out_len) + " floats; the batch needs " +
                                            std::to_string((long long)need) + " ([n_lines][3][H][wmax])");
    if (rgb_len > 0 && !rgb) return fail(RH_ERR_INVALID_ARG, "null pixel buffer");
    // contiguous line shards of equal size (every line has the same output size), one per device
    const int nd = (int)ctx->slots.size();
    return run_shards(nd, [&](int d, int slot) -> int {
        return rec_host_on_slot(ctx, slot, rgb, rgb_offsets, widths, heights, n_lines * d / nd, n_lines * (d + 1) / nd,
                                b, out);
    });
}

int rh_rec_preprocess_device(rh_ctx* ctx, int slot, const uint8_t* d_rgb, int64_t rgb_len, const int64_t* rgb_offsets,
                             const uint32_t* widths, const uint32_t* heights, int64_t n_lines, uint32_t target_h,
                             uint32_t max_w, float* d_out, int64_t out_len, uint32_t* out_widths, uint32_t* out_wmax,
                             void* stream) {
    if (int rc = check_ctx(ctx)) return rc;
    if (slot < 0 || slot >= (int)ctx->slots.size()) return fail(RH_ERR_INVALID_ARG, "slot out of range");
    if (rgb_len < 0) return fail(RH_ERR_INVALID_ARG, "negative pixel buffer length");
    if (n_lines > 0 && !rgb_offsets) return fail(RH_ERR_INVALID_ARG, "null crop offsets");
    RecBatch b;
    if (int rc = rec_validate(rgb_offsets, widths, heights, n_lines, target_h, max_w, rgb_len, b)) return rc;
    if (out_widths && n_lines > 0) std::memcpy(out_widths, b.out_w.data(), (size_t)n_lines * sizeof(uint32_t));
    if (out_wmax) *out_wmax = b.wmax;
    if (n_lines == 0) return RH_OK;
    const long double need = (long double)n_lines * 3.0L * b.out_h * b.wmax;
    if (!d_out || (long double)out_len < need)
        return fail(RH_ERR_INVALID_ARG, "output holds " + std::to_string(out_len) + " floats; the batch needs " +
                                            std::to_string((long long)need) + " ([n_lines][3][H][wmax])");
    if (rgb_len > 0 && !d_rgb) return fail(RH_ERR_INVALID_ARG, "null pixel buffer");
    if ((long double)n_lines * b.out_h > 2147483647.0L)
        return fail(RH_ERR_UNSUPPORTED, "n_lines x target height above 2^31 - 1; split the batch");
    std::vector<rh::RecLine> lines;
    long long n_coords, n_wts;
    int span_cap, meta_cap;
    rec_describe(rgb_offsets, widths, heights, 0, n_lines, b, 0, lines, n_coords, n_wts, span_cap, meta_cap);
    Slot& s = *ctx->slots[slot];
    std::lock_guard<std::mutex> lock(s.mu);
    RH_CUDA(cudaSetDevice(s.device));
    cudaStream_t st = (cudaStream_t)stream;
    if (int rc = rec_tables(s, st, n_lines, n_coords, n_wts)) return rc;
    rh::RecParams p{};
    p.rgb = d_rgb;
    p.lines = (const rh::RecLine*)s.pre_lines.p;
    p.n_lines = n_lines;
    p.out_h = (int)b.out_h;
    p.wmax = (int)b.wmax;
    p.span_cap = span_cap;
    p.meta_cap = meta_cap;
    p.coords = (int2*)s.pre_coords.p;
    p.wts = (float*)s.pre_wts.p;
    p.out = d_out;
    p.inv = 1.0f / 127.5f;
    p.status = s.d_status;
    RH_CUDA(cudaMemcpyAsync(s.pre_lines.p, lines.data(), (size_t)n_lines * sizeof(rh::RecLine), cudaMemcpyHostToDevice,
                            st));
    RH_CUDA(rh::launch_rec_weights(p, st));
    RH_CUDA(rh::launch_rec_resize(p, 0, n_lines, st));
    RH_CUDA(cudaEventRecord(s.pre_done, st));
    s.launches += 2;
    return RH_OK;
}

}  // extern "C"
