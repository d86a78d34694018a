// vw_internal.h -- launch-parameter layout shared by the C-ABI host code (vw_api.cpp) and the sampler kernel
// (vw_sampler.cu).  Not part of the public ABI.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace vw {

constexpr int kMaxSegments = 8;        // == VW_MAX_SEGMENTS
constexpr int kInlineOptions = 32;     // option tables up to this size travel in the kernel parameters
constexpr int kThreads = 128;          // one warp-group per logits row
constexpr int kWarps = kThreads / 32;
constexpr int kRegElems = 24;          // elements per thread held in registers: rows of <= 3072 active ids
constexpr int kSmallK = 64;            // top-k <= kSmallK uses the candidate path
constexpr int kCandCap = 128;          // candidate buffer entries (one warp sorts 4 per lane)
constexpr int kMaxStageLogitBytes = 64 * 1024;
constexpr int kMaxHistStage = 4096;    // history ids staged per row; longer histories stream the rest
constexpr int kStages = 3;

// Counters of rows by path (vw_stats field order).
enum : int {
    kStatGreedy = 0,
    kStatFast = 1,             // candidate rows decided in parallel by the chain warp
    kStatFastReplayed = 2,     // candidate rows replayed in the reference's order
    kStatGeneral = 3,          // whole-row rows decided in parallel
    kStatGeneralReplayed = 4,  // whole-row rows replayed in the reference's order
    kStatLarge = 5,            // rows of more than 3072 active ids (always replayed)
    kStatOverflow = 6,         // candidate-eligible rows that took the whole-row path
    kStatThresholdMiss = 7,    // candidate rows whose carried threshold missed (lowered or rebuilt)
    kNumStats = 9,             // slot 8 is vw_stats.h2d_bytes, kept on the host
};

// Error bits latched in the device error word.
enum : unsigned {
    kErrHistRange = 1u,   // a history id outside [0, V)
    kErrTimeout = 2u,     // an mbarrier wait gave up
    kErrBadOption = 4u,   // a row's option index outside the table
    kErrHistOffsets = 8u, // a row's history offsets negative or decreasing (the row is sampled without history)
    kErrCodeRange = 16u,  // a frame code outside its codebook (vw_frame_embedding; the row is not written)
};

constexpr int kMaxCodeGroups = 16;     // codebooks per frame (Qwen3TtsConfig.NumCodeGroups)

// The next talker input of n_rows sequences: sum of the frame's codebook embeddings plus the text row (vw_embed.cu).
cudaError_t launch_frame_embedding(const int32_t* codes, int n_rows, int n_groups, int hidden,
                                   const uint16_t* const* tables, int vocab, int cp_vocab, const float* text,
                                   float* out, unsigned* err, cudaStream_t stream);

struct DevOptions {       // same layout as vw_options
    int32_t do_sample;
    int32_t top_k;
    float top_p;
    float temperature;
    float rep_penalty;
};

struct DevSegment {
    const void* logits;
    const int64_t* hist_offsets;
    const int32_t* hist_ids;
    const int32_t* steps;
    const int32_t* opt_index;
    const double* uniforms;
    int32_t* out_ids;
    double* out_probs;
    int64_t row_stride;   // elements
    int32_t row_begin;    // first global row of the segment
    int32_t n_rows;
    int32_t vocab;
    int32_t dtype;        // 0 f32, 1 bf16
    int32_t kind;         // 0 talker, 1 sub
    int32_t sup_lo, sup_hi, eos, min_new;   // talker suppress mask (clamped to [0, vocab]); lo == hi: none
    int32_t bulk_ok;      // rows are 16-byte aligned with 16-byte multiple sizes: bulk copies allowed
    int32_t hist_aligned; // hist_ids is 16-byte aligned
    // ---- the row's active vectors (16 bytes each) for the warp-per-row kernel, in global vector indices:
    //      part A [0, va), the EOS vector eosv (or -1) when EOS lies inside the skipped suppress span, part C
    //      [c0, c0 + vc).  Vectors [spec_a, spec_b] of parts A and C hold suppressed ids (partial vectors at the
    //      span's edges, or a span too short to skip); they are always examined element by element.
    int32_t vsh;          // log2 of the ids per vector (2 fp32, 3 bf16)
    int32_t va, c0, vc, eosv, spec_a, spec_b;
    int32_t cpl_a, cpl_c; // vectors per lane of parts A and C (lane l takes the contiguous vectors l * cpl ...)
    int32_t rw_ok;        // rows of this segment fit the warp-per-row kernel (aligned, <= 32 vectors per lane)
    // ---- device-resident batches (vw_batch_*): histories in place, inactive rows skipped
    const int32_t* hist_lens;   // non-null: row r's history is hist_ids[r * hist_stride, + hist_lens[r]) (no CSR)
    int64_t hist_stride;
    const int32_t* active;      // non-null: rows with active[r] == 0 are not sampled (their id is -1)
};

// Fills the warp-per-row layout fields of a segment whose other fields are set.
void fill_row_layout(DevSegment& d);

// Row r's history span [hb, he) in hist_ids: CSR offsets, or the strided layout of a device-resident batch.
__host__ __device__ inline bool row_history(const DevSegment& sg, int local, int64_t& hb, int64_t& he) {
    if (sg.kind != 0) return false;
    if (sg.hist_lens) {
        hb = static_cast<int64_t>(local) * sg.hist_stride;
        he = hb + sg.hist_lens[local];
        return true;
    }
    if (!sg.hist_offsets) return false;
    hb = sg.hist_offsets[local];
    he = sg.hist_offsets[local + 1];
    return true;
}

// ---- device-resident generation state (vw_batch.cu)
struct DotNetRngState {        // System.Random(int): the subtractive generator's table and its two indices
    int32_t seed[56];
    int32_t inext, inextp;
};
struct BatchDevice {
    int32_t n_slots, max_history, eos;
    int32_t* history;          // [n_slots, max_history] the talker ids generated so far (Active.History)
    int32_t* hist_len;         // [n_slots]
    int32_t* step;             // [n_slots] Active.Step
    int32_t* active;           // [n_slots] 1 while the slot's job runs
    int32_t* max_new;          // [n_slots] GenerationOptions.MaxNewTokens
    int32_t* opt_talker;       // [n_slots] the slot's index into each talker step's options table
    int32_t* opt_sub;          // [n_slots] ... into each sub-talker step's options table
    DotNetRngState* rng_talker;   // [n_slots] Sampler(Seed)
    DotNetRngState* rng_sub;      // [n_slots] Sampler(Seed + 1)
    int32_t* codes;               // [n_slots, kMaxCodeGroups] the frame being built (keepFrames); codes[s][0] is -1
                                  // unless slot s continues past its last talker step
};
// One NextDouble() into uniforms[s] for every active slot whose option samples (which: 0 talker, 1 sub-talker).
cudaError_t launch_batch_draw(const BatchDevice& b, int which, const DevOptions* opts, int n_opts, double* uniforms,
                              cudaStream_t stream);
// Where a slot's gathered embedding row goes: out[s] (row pitch out_stride floats) = bf16 -> fp32 of table row code
// (table [table_rows, hidden] bf16 bits, hidden a multiple of 8, 16-byte aligned rows).
struct EmbedOut {
    const uint16_t* table;
    int table_rows, hidden;
    float* out;
    int64_t out_stride;
};
// Appends ids[s] to every active slot's history, then retires the slot (EOS or last step) or advances its step;
// records code 0 of the frame of every slot that continues (-1 for the others) and, with `e`, gathers that code's
// row of e->table for it.  err collects kErrCodeRange.
cudaError_t launch_batch_commit(const BatchDevice& b, const int32_t* ids, int32_t* out_done, const EmbedOut* e,
                                unsigned* err, cudaStream_t stream);
// codes[s][group] = ids[s] for every slot (a code-predictor group's ids; -1 where the slot did not sample) and, with
// `e`, the row of e->table for each slot whose frame goes on.
cudaError_t launch_batch_record_codes(const BatchDevice& b, const int32_t* ids, int group, const EmbedOut* e,
                                      unsigned* err, cudaStream_t stream);
// The row of e.table at codes[s][group] for every continuing slot (TalkerModel.CodecEmbedding for group 0,
// CodePredictorEmbedding for groups 1..15); other rows are left alone.
cudaError_t launch_batch_code_embedding(const BatchDevice& b, int group, const EmbedOut& e, unsigned* err,
                                        cudaStream_t stream);

struct LaunchParams {
    DevSegment seg[kMaxSegments];
    DevOptions inl_opts[kInlineOptions];
    float inl_inv_t[kInlineOptions];      // fp32(1 / temperature) of each inline option (Sampler.cs:39)
    double inl_pen_rcp[kInlineOptions];   // RN64(1 / repetition_penalty) of each inline option
    const DevOptions* dev_opts;   // used when n_opts > kInlineOptions
    int32_t n_opts;
    int32_t n_segs;
    int32_t total_rows;
    int32_t n_stages;
    int32_t stage_logit_bytes;    // multiple of 16
    int32_t stage_hist_cap;       // ids per stage, multiple of 4
    int32_t flag_bytes;           // history flag map: a byte per id, vmax rounded up to 16
    int32_t vmax;
    unsigned* err;
    int32_t* deferred_rows;       // rows the warp-per-row kernel leaves to the whole-row kernel (total_rows entries)
    uint32_t* deferred_count;     // their number (the whole-row kernel resets it to 0 when it is done)
    uint32_t* done_count;         // whole-row kernel CTAs finished (reset with deferred_count)
    unsigned long long* stats;    // kNumStats counters (nullable)
    int32_t force_exact;          // replay every sampled row in the reference's order (test hook)
    char* gscratch;               // large-path scratch, gscratch_stride bytes per CTA
    int64_t gscratch_stride;
    unsigned long long* guess_seed;   // kSeedSlots candidate thresholds per segment carried across calls, each
                                      // float bits << 32 | option; nullable (any value is safe: it only saves work
                                      // when it fits)
    uint64_t wait_ns;             // bound of every mbarrier wait without progress
    int32_t test_stall_row;       // test hook: the whole-row kernel's producer withholds this row's stage (-1: none)
};

constexpr uint64_t kWaitLimitNs = 2000000000ull;   // default wait bound: 2 s without progress
constexpr uint64_t kTestWaitLimitNs = 1000000ull;  // with the stall test hook: 1 ms

// Dynamic shared memory the whole-row kernel needs for `p`.
size_t sampler_smem_bytes(const LaunchParams& p);
// Global scratch bytes per CTA for rows of up to `vmax` ids.
int64_t sampler_gscratch_stride(int vmax);

struct LaunchPlan {
    int grid;              // warp-per-row kernel CTAs (every row)
    int grid_general;      // whole-row kernel CTAs (the deferred rows)
    size_t smem_cand;      // dynamic shared memory of each
    size_t smem_general;
};
// Picks p.n_stages and both grids for `sm_count` SMs on the current device (whole-row grid <= max_grid_general).
// False when a row does not fit in shared memory.
bool plan_launch(LaunchParams& p, int sm_count, int max_grid_general, LaunchPlan* plan);
// The warp-per-row kernel over every row, then the whole-row kernel over the rows it deferred (stream-ordered).
cudaError_t launch_sampler(const LaunchParams& p, const LaunchPlan& plan, cudaStream_t stream);

// ---- fixed scratch of vw_sample_static: one file-scope device array per device, no allocation.
// Layout: the error word, the two deferred-list counters and the two row-scheduling counters at offset 0 (zeroed
// before every call), the carried
// candidate thresholds (one per segment) at kStaticGuessOffset, the deferred
// rows at kStaticRowsOffset, then one kStaticCtaStride slice per whole-row CTA at kStaticScratchOffset.
constexpr int kStaticMaxRows = 65536;       // rows per call (all segments)
constexpr int kStaticMaxVocab = 4096;       // ids per row (a power of two >= kRegElems * kThreads)
constexpr int kStaticGeneralCtas = 148;     // whole-row kernel CTAs (one per B200 SM)
constexpr int kSeedSlots = 32;                // carried thresholds per segment (one per warp lane)
constexpr int64_t kStaticGuessOffset = 256;   // kMaxSegments * kSeedSlots carried thresholds
constexpr int64_t kStaticRowsOffset = 4096;
static_assert(kStaticGuessOffset + 8 * kMaxSegments * kSeedSlots <= kStaticRowsOffset, "static scratch layout");
constexpr int64_t kStaticScratchOffset = kStaticRowsOffset + 4 * static_cast<int64_t>(kStaticMaxRows);
// sampler_gscratch_stride(kStaticMaxVocab): 12 bytes per id plus a 16-byte sort slot per id
constexpr int64_t kStaticCtaStride = (static_cast<int64_t>(kStaticMaxVocab) * 28 + 255) / 256 * 256;
constexpr int64_t kStaticBytes = kStaticScratchOffset + kStaticGeneralCtas * kStaticCtaStride;   // ~16.4 MiB
// Device address of this device's array (the device must be current); cudaGetSymbolAddress's status.
cudaError_t static_scratch_address(char** ptr);

// The sampler's exp and CUDA's exp over n device doubles (see vw_exp_diagnostic).
cudaError_t launch_exp_diagnostic(const double* x, int64_t n, double* y_libm, double* y_cuda, int sm_count,
                                  cudaStream_t stream);

// logits[M, N] (fp32, row pitch ldo) = A[M, K] x B[N, K]^T, A and B bf16 row-major (pitches lda, ldb elements,
// multiples of 8), on the tcgen05 tensor cores (vw_head.cu).  err collects kErrTimeout.
cudaError_t launch_head_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, float* out,
                             int64_t ldo, unsigned* err, cudaStream_t stream);

// Sampler.ApplyRepetitionPenalty on one device row, in place.
cudaError_t launch_apply_penalty(float* logits, int vocab, const int32_t* hist, int64_t hist_len, float penalty,
                                 unsigned* err, cudaStream_t stream);

}  // namespace vw
