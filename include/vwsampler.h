/*
 * vwsampler.h -- C ABI of the B200 (sm_100a) token sampler for voxwerk's Qwen3-TTS generation loop.
 *
 * The library replaces, with one batched GPU call, the per-row sampling block that voxwerk runs on the CPU:
 *
 *   talker rows (codebook 0, V = 3072)       src/Voxwerk/Talker/TalkerGenerator.cs:369-373 (GenerateBatch)
 *                                            src/Voxwerk/Talker/TalkerGenerator.cs:246-249 (Generate)
 *     Sampler.ApplyRepetitionPenalty(lg, history, RepetitionPenalty)   Sampler.cs:25-33
 *     suppress ids [V-1024, V) except EOS; EOS too while t < 2         TalkerGenerator.cs:247-248 / :371-372
 *     Sampler.Select(lg, options.Talker)                               Sampler.cs:35-88
 *   sub-talker rows (codebooks 1..15, V = 2048)
 *     Sampler.Select(cpLogits[row], options.SubTalker)                 TalkerGenerator.cs:420 / :268
 *
 * The reference has no FFI for this path (Sampler is a sealed C# class called directly); the entry points
 * below are what its P/Invoke layer would bind.  Every struct is plain-old-data and blittable.
 *
 * Random numbers stay with the caller: each sampled row takes one uniform, the value the reference's
 * Sampler._rng.NextDouble() would return at Sampler.cs:77 (talker rows from Random(Seed), sub-talker rows from
 * Random(Seed + 1), TalkerGenerator.cs:217-218 / :345-346).  Greedy rows take no draw and ignore their slot.
 *
 * Threading: a handle is bound to one CUDA device and must not be used by two host threads at once (like
 * Sampler, whose System.Random is not thread-safe).  Use one handle per GPU per host thread.
 */
#ifndef VWSAMPLER_H
#define VWSAMPLER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VW_ABI_VERSION 1

/* Status codes.  No C++ exception crosses the ABI. */
typedef enum vw_status {
    VW_OK = 0,
    VW_ERR_INVALID_ARG = 1,  /* bad pointer, size, dtype, option (e.g. Temperature <= 0 with DoSample) */
    VW_ERR_OUT_OF_RANGE = 2, /* a history id outside [0, V): the reference throws at Sampler.cs:30 */
    VW_ERR_CUDA = 3,         /* a CUDA runtime error; see vw_last_error() */
    VW_ERR_TIMEOUT = 4,      /* a bounded wait inside the kernel gave up; results are not valid */
    VW_ERR_NO_DEVICE = 5     /* no CUDA device with that ordinal, or not an sm_100 device */
} vw_status;

typedef enum vw_dtype { VW_F32 = 0, VW_BF16 = 1 } vw_dtype;

/* Row kinds.  TALKER rows get the repetition penalty and the suppress mask; SUB rows get neither. */
typedef enum vw_row_kind { VW_ROWS_TALKER = 0, VW_ROWS_SUB = 1 } vw_row_kind;

/* Where the pointers of a call live.  DEVICE: every array is device memory on the handle's device and the call
 * is stream-ordered.  HOST: every array is host memory; the library copies inputs to the device and the ids
 * back, and returns when they are written. */
typedef enum vw_mem { VW_MEM_DEVICE = 0, VW_MEM_HOST = 1 } vw_mem;

/* One stage's decoding settings: SamplingOptions (Sampler.cs:4-13) plus GenerationOptions.RepetitionPenalty
 * (TalkerGenerator.cs:11), which only talker rows use.  Defaults: {1, 50, 1.0f, 0.9f, 1.05f}. */
typedef struct vw_options {
    int32_t do_sample;          /* SamplingOptions.DoSample (0 = argmax, Sampler.cs:37) */
    int32_t top_k;              /* SamplingOptions.TopK; <= 0 or >= V disables the cut (Sampler.cs:42) */
    float top_p;                /* SamplingOptions.TopP; >= 1 disables the cut (Sampler.cs:62) */
    float temperature;          /* SamplingOptions.Temperature; must be > 0 when do_sample */
    float repetition_penalty;   /* GenerationOptions.RepetitionPenalty; 1.0f disables (Sampler.cs:27) */
} vw_options;

/* A block of rows that share vocabulary size, dtype and kind.  A call takes up to VW_MAX_SEGMENTS segments, so
 * one launch can hold the talker rows and the sub-talker rows of a frame. */
#define VW_MAX_SEGMENTS 8

typedef struct vw_segment {
    const void* logits;          /* [n_rows, row_stride] elements of `dtype`; read-only */
    int64_t row_stride;          /* elements between consecutive rows (>= vocab) */
    int32_t n_rows;
    int32_t vocab;               /* V: 3072 talker (Qwen3TtsConfig.cs:28), 2048 code predictor (:49) */
    int32_t dtype;               /* vw_dtype */
    int32_t kind;                /* vw_row_kind */
    /* ---- talker rows only (ignored for SUB rows) ---- */
    const int64_t* hist_offsets; /* [n_rows + 1] CSR offsets into hist_ids; NULL = every history empty */
    const int32_t* hist_ids;     /* ids generated so far by each row's sequence (Active.History) */
    const int32_t* steps;        /* [n_rows] generation step t (Active.Step); NULL = every row at t >= min_new_tokens */
    int32_t suppress_lo;         /* ids [suppress_lo, suppress_hi) except eos_id become -inf; voxwerk: V - 1024 */
    int32_t suppress_hi;         /* voxwerk: V */
    int32_t eos_id;              /* codec EOS, Qwen3TtsConfig.cs:34: 2150 */
    int32_t min_new_tokens;      /* EOS is suppressed while t < min_new_tokens; voxwerk: 2 */
    int32_t max_hist_len;        /* optional hint: the longest history in the segment (0 = unknown) */
    /* ---- all rows ---- */
    const int32_t* opt_index;    /* [n_rows] index into the options table; NULL = options[0] for every row */
    const double* uniforms;      /* [n_rows] NextDouble() per row; may be NULL only if every row is greedy */
    int32_t* out_ids;            /* [n_rows] sampled token ids */
    double* out_probs;           /* optional [n_rows, vocab]: the probabilities the draw scanned (after top-k,
                                    softmax, top-p and renormalisation), 0 for every other id; NULL = none */
} vw_segment;

/* Rows sampled per path since the handle was created (or last reset).  Every path returns the reference's id;
 * the counters show where the time goes.  "replayed" rows had a top-p or draw decision within the proven error
 * band of the parallel sums and were recomputed in the reference's sequential order. */
typedef struct vw_stats {
    uint64_t rows_greedy;            /* DoSample == false: argmax */
    uint64_t rows_fast;              /* top-k <= 64 rows decided from their candidates in parallel */
    uint64_t rows_fast_replayed;     /* top-k <= 64 rows replayed in the reference's order */
    uint64_t rows_general;           /* whole-row rows (top-k off / larger K / candidate overflow), parallel */
    uint64_t rows_general_replayed;  /* whole-row rows replayed in the reference's order */
    uint64_t rows_large;             /* rows of more than 3072 active ids (always replayed) */
    uint64_t rows_overflow;          /* top-k <= 64 rows whose candidates overflowed (counted in rows_general*) */
    uint64_t rows_threshold_miss;    /* top-k <= 64 rows whose carried candidate threshold missed: lowered (a few
                                        candidates short) or rebuilt from the row, then collected once more (extra
                                        work, same result; a row still missing counts in rows_overflow) */
    uint64_t h2d_bytes;              /* bytes VW_MEM_HOST calls copied host -> device (inputs only: the logit
                                        columns of a suppressed span are not copied, no kernel reads them) */
} vw_stats;

typedef struct vw_handle vw_handle;

/* Library version string, e.g. "vwsampler 1.0 (sm_100a)". */
const char* vw_version(void);

/* Human-readable name of a status code. */
const char* vw_status_string(vw_status status);

/* Creates a handle on CUDA device `device`.  Replaces `new Sampler(seed)` (Sampler.cs:21) as the per-worker
 * object; the RNG stays with the caller. */
vw_status vw_create(int32_t device, vw_handle** out_handle);

/* Frees the handle and all device memory it owns.  Safe on NULL. */
vw_status vw_destroy(vw_handle* handle);

/* Message of the last error on this handle ("" if none).  Valid until the next call on the handle. */
const char* vw_last_error(const vw_handle* handle);

/*
 * Samples one token id for every row of every segment.  Replaces, for a whole batch, the per-row sequence
 * ApplyRepetitionPenalty -> suppress mask -> Select of TalkerGenerator.cs:366-385 (talker rows) and the per-row
 * SubSampler.Select of TalkerGenerator.cs:419-420 (sub-talker rows); results are the ids those loops return.
 *
 * options / n_options: host array (always host memory), indexed by each row's opt_index.
 * mem: VW_MEM_DEVICE or VW_MEM_HOST (see vw_mem).
 * stream: a cudaStream_t for VW_MEM_DEVICE calls, or NULL.  With NULL the call runs on the handle's stream and
 *   returns after the ids are written, reporting device-side errors.  With a stream the call is enqueued and
 *   returns at once; device-side errors (history id out of range, timeout) are reported by the next
 *   vw_synchronize() on that stream.  VW_MEM_HOST calls are always synchronous.
 */
vw_status vw_sample(vw_handle* handle, const vw_segment* segments, int32_t n_segments,
                    const vw_options* options, int32_t n_options, int32_t mem, void* stream);

/* Waits for work enqueued on `stream` (NULL = the handle's stream) and returns, then clears, any device-side
 * error latched by earlier calls. */
vw_status vw_synchronize(vw_handle* handle, void* stream);

/* Copies the per-path row counters into *out (after any vw_synchronize the caller needs); `reset` != 0 clears
 * them.  Setting the environment variable VW_FORCE_EXACT=1 before vw_create makes every sampled row take the
 * sequential replay (a test hook; results are identical, only slower).  VW_TEST_STALL_ROW=r before vw_create makes
 * the handle's first vw_sample call withhold row r's input stage inside the whole-row kernel (row r must be one that
 * kernel takes, e.g. a row with top-k off), with the kernel's bounded waits cut to 1 ms: that call returns
 * VW_ERR_TIMEOUT (a test hook for the timeout path; later calls are unaffected). */
vw_status vw_get_stats(vw_handle* handle, vw_stats* out, int32_t reset);

/*
 * vw_sample for callers that cannot allocate device memory: a process whose memory is all held by its own pool
 * (a serving engine that reserves the free HBM up front), a host runtime whose binding exposes no device
 * allocator, or code inside a region where allocation is forbidden.  No counterpart in the reference: voxwerk
 * samples on the CPU and manages no device memory.  Results are vw_sample's.
 *
 * The call takes no handle and allocates nothing.  Its scratch is one fixed device array per device (about
 * 16.4 MiB, built into the library, loaded on first use, held until the process exits); every call looks up that
 * array's address on the device.  The call is synchronous: it ends by synchronizing its stream and reading the
 * error word back, so it cannot be captured into a CUDA graph.
 *
 * Limits (larger requests fail with VW_ERR_INVALID_ARG and a message): at most 65536 rows per call over all
 * segments, vocab <= 4096, n_options <= 32.  Every array is device memory of `device` (as VW_MEM_DEVICE; each
 * non-NULL pointer is checked, and a host or foreign pointer fails with VW_ERR_INVALID_ARG); there is no
 * host-memory mode.
 *
 * stream: a cudaStream_t of `device`, or NULL for the default stream.  The call returns after the stream has
 *   finished it, reporting device-side errors in its status.
 * err_msg / err_msg_len: optional buffer for a NUL-terminated message ("" on success).
 *
 * Calls on one device share the array: two calls that overlap in time (from two host threads, say) race and
 * both results are undefined.  Serialise them per device.
 */
vw_status vw_sample_static(int32_t device, const vw_segment* segments, int32_t n_segments,
                           const vw_options* options, int32_t n_options, void* stream, char* err_msg,
                           int32_t err_msg_len);

/*
 * Device-resident generation state: TalkerGenerator.GenerateBatch's per-job state (TalkerGenerator.cs:322-455) kept
 * in device memory, one slot per job, so that a generation step sends only logits and reads only ids.  Per slot: the
 * talker ids generated so far (Active.History, :304), the step (Active.Step), MaxNewTokens, the job's two samplers
 * (Sampler(Seed) for the talker and Sampler(Seed + 1) for the sub-talker, :345-346, System.Random restated on the
 * device; their NextDouble() draws replace the per-row uniforms) and whether the job still runs.
 *
 * Row r of a step's logits belongs to slot r (row_stride elements apart, device memory).  Finished slots are not
 * sampled (their id is -1) and draw nothing, like the retired jobs the reference drops from its active list.
 * Steps are stream-ordered on `stream` (NULL: the handle's stream, and the call returns after the step with any
 * device-side error); n_options <= 32.  A batch belongs to its handle and its host thread.
 */
typedef struct vw_batch vw_batch;

typedef struct vw_slot_config {
    int32_t talker_option;    /* index of the job's talker options (+ RepetitionPenalty) in each talker step's table */
    int32_t sub_option;       /* index of the job's sub-talker options in each sub-talker step's table */
    int32_t max_new_tokens;   /* GenerationOptions.MaxNewTokens */
    int32_t seed;             /* GenerationOptions.Seed, when seeded != 0 */
    int32_t seeded;           /* 0: an unseeded job (new Random(); the draws are not reproducible, as in voxwerk) */
} vw_slot_config;

/* n_slots jobs at most; vocab, eos_id, min_new_tokens and the suppress span as in vw_segment (voxwerk: 3072, 2150,
 * 2, [2048, 3072)); max_history >= each job's initial history length + max_new_tokens. */
vw_status vw_batch_create(vw_handle* handle, int32_t n_slots, int32_t vocab, int32_t max_history, int32_t eos_id,
                          int32_t min_new_tokens, int32_t suppress_lo, int32_t suppress_hi, vw_batch** out_batch);
/* Frees the batch.  vw_destroy of its handle releases the device memory of every batch still alive on it; the
 * caller then still calls vw_batch_destroy (which only frees the host object), and every other call on such a batch
 * returns VW_ERR_INVALID_ARG. */
vw_status vw_batch_destroy(vw_batch* batch);

/* Starts a job in `slot` (the slot refill of TalkerGenerator.cs:336-358): step 0, running, the two samplers seeded,
 * and the talker history set to history[0..history_len) (host memory; voxwerk starts from an empty one). */
vw_status vw_batch_start(vw_batch* batch, int32_t slot, const vw_slot_config* config, const int32_t* history,
                         int32_t history_len);

/* Ends the job in `slot` early (the slot is not sampled again until the next vw_batch_start). */
vw_status vw_batch_stop(vw_batch* batch, int32_t slot);

/*
 * One talker step for every running slot (TalkerGenerator.cs:366-385): repetition penalty over the slot's history,
 * suppress mask, Select with the slot's options and its talker sampler's draw; then the id is appended to the
 * history and the job ends when the id is EOS or its step is MaxNewTokens - 1 (out_done[slot] = 1), else its step
 * advances.  logits: [n_slots, row_stride] of dtype; out_ids / out_done (nullable): [n_slots] int32, device memory.
 */
vw_status vw_batch_talker_step(vw_batch* batch, const void* logits, int64_t row_stride, int32_t dtype,
                               const vw_options* options, int32_t n_options, int32_t* out_ids, int32_t* out_done,
                               void* stream);

/* One code-predictor group for every running slot (TalkerGenerator.cs:419-420): Select with the slot's sub-talker
 * options and its sub-talker sampler's draw.  logits: [n_slots, row_stride], `vocab` ids (voxwerk: 2048). */
vw_status vw_batch_sub_step(vw_batch* batch, const void* logits, int64_t row_stride, int32_t vocab, int32_t dtype,
                            const vw_options* options, int32_t n_options, int32_t* out_ids, void* stream);

/* A slot's step, history length and running flag (after the steps enqueued so far; synchronizes). */
vw_status vw_batch_query(vw_batch* batch, int32_t slot, int32_t* step, int32_t* history_len, int32_t* active);

/*
 * The per-frame loop of GenerateBatch (TalkerGenerator.cs:362-439) on the device, around the caller's transformer
 * steps.  The batch keeps the frame being built, codes[n_slots][16] (keepFrames, :382, :420): a talker step records
 * code 0 of every slot that goes on to the code predictor and -1 for the others (idle, or retired at this step by
 * EOS or MaxNewTokens); sub-talker head step `group` records codebook `group`.  Per frame:
 *   vw_batch_talker_head_step                 codebook 0 from the talker's last hidden rows      (:366-385, :443)
 *                                             + CodecEmbedding(code0), the code predictor's 2nd input row (:411)
 *   for group = 1..15:
 *     vw_batch_sub_head_step(group)           CodePredictorHead(group) + SubSampler.Select          (:418-420)
 *                                             + CodePredictorEmbedding(group, code), the next input (:422)
 * (the gathers ride along with a vw_embed_out; vw_batch_code_embedding does them alone)
 *   vw_batch_frame_embedding                  FrameEmbedding(frame) + text, the next talker input (:428-439)
 * Head steps: hidden [n_slots, hidden_size] and weight [vocab, hidden_size] bf16 as in vw_head_logits (rows of
 * idle slots are multiplied but not sampled); the logits live in a buffer of the batch.  The ids come out as in
 * vw_batch_talker_step / vw_batch_sub_step (out_ids [n_slots], -1 for slots that did not sample).  All calls are
 * stream-ordered and allocate nothing after a batch's first head step of the largest vocab, so a frame can be
 * captured in a CUDA graph.
 */
/* Where a head step also writes the next input row of each slot whose frame goes on: out[s] (row pitch out_stride
 * floats) = bf16 -> fp32 of table[code] -- CodecEmbedding(code0) for the talker step (TalkerGenerator.cs:411),
 * CodePredictorEmbedding(group, code) for a sub-talker step (:422).  table: [table_rows, hidden] bf16 bits, hidden a
 * multiple of 8 (the talker's hidden size in voxwerk, which the code predictor's embeddings share); 16-byte aligned
 * device memory.  The same as a vw_batch_code_embedding call after the step, in the step's last kernel. */
typedef struct vw_embed_out {
    const void* table;
    int32_t table_rows;
    int32_t hidden;
    float* out;
    int64_t out_stride;
} vw_embed_out;

vw_status vw_batch_talker_head_step(vw_batch* batch, const void* hidden, int64_t hidden_stride, int32_t hidden_size,
                                    const void* weight, int64_t weight_stride, const vw_options* options,
                                    int32_t n_options, int32_t* out_ids, int32_t* out_done,
                                    const vw_embed_out* embed /* NULL: no gather */, void* stream);
vw_status vw_batch_sub_head_step(vw_batch* batch, int32_t group, const void* hidden, int64_t hidden_stride,
                                 int32_t hidden_size, const void* weight, int64_t weight_stride, int32_t vocab,
                                 const vw_options* options, int32_t n_options, int32_t* out_ids,
                                 const vw_embed_out* embed /* NULL: no gather */, void* stream);
/* out[s] (row pitch out_stride floats) = bf16 -> fp32 of table row codes[s][group] for every slot whose frame goes
 * on (codes[s][0] >= 0); other rows are left alone.  table: [table_rows, hidden] bf16 bits (group 0: the talker
 * codec embedding, vocab rows; group g: code-predictor embedding g-1).  A code outside the table returns
 * VW_ERR_OUT_OF_RANGE. */
vw_status vw_batch_code_embedding(vw_batch* batch, int32_t group, const void* table, int32_t table_rows,
                                  int32_t hidden, float* out, int64_t out_stride, void* stream);
/* vw_frame_embedding over the batch's codes table (n_slots rows, 16 groups); slots with codes[s][0] == -1 are
 * skipped. */
vw_status vw_batch_frame_embedding(vw_batch* batch, int32_t hidden, const uint16_t* codec_embedding,
                                   const uint16_t* const* cp_embeddings, int32_t cp_vocab, const float* text,
                                   float* out, void* stream);
/* Copies the codes table [n_slots, 16] int32 to host memory (after the handle's stream drains). */
vw_status vw_batch_get_codes(vw_batch* batch, int32_t* out);

/*
 * The next talker input of n_rows sequences once their frames are sampled (TalkerGenerator.cs:428-439):
 *   out[r] = FrameEmbedding(codes[r]) + text[r]     (TalkerModel.cs:114-118, TalkerGenerator.cs:437-438)
 * i.e. the bf16 row codes[r][0] of the talker codec embedding widened to fp32, plus for g = 1..n_groups-1 the row
 * codes[r][g] of code-predictor embedding g-1, plus the text row, each addition rounded once in that order, so the
 * result equals the reference's bit for bit.
 * codes: [n_rows, n_groups] int32 (n_groups <= 16; voxwerk: 16); a row whose codes[r][0] is -1 (a finished slot of
 *   vw_batch_talker_step) is skipped and its output left as it was.
 * codec_embedding: [vocab, hidden] bf16 bits; cp_embeddings: host array of n_groups-1 device pointers, each
 *   [cp_vocab, hidden] bf16 bits (voxwerk: 3072 / 2048 ids, hidden 1024, a multiple of 8 here).
 * text: [n_rows, hidden] fp32 (the step's trailing text row or tts_pad per sequence), or NULL to add nothing.
 * out: [n_rows, hidden] fp32.  Device memory, 16-byte aligned.  A code outside its codebook returns
 * VW_ERR_OUT_OF_RANGE (the reference throws, TalkerModel.cs:99, :106).  stream as in vw_sample.
 */
vw_status vw_frame_embedding(vw_handle* handle, const int32_t* codes, int32_t n_rows, int32_t n_groups,
                             int32_t hidden, const uint16_t* codec_embedding, int32_t vocab,
                             const uint16_t* const* cp_embeddings, int32_t cp_vocab, const float* text, float* out,
                             void* stream);

/*
 * The vocabulary head alone: out_logits[n_rows, vocab] (fp32, row pitch vocab) = hidden x weight^T -- the logits
 * TalkerModel.CodecHead (TalkerModel.cs:133) and CodePredictorHead (:136-137) produce -- on the tcgen05 tensor cores
 * (bf16 inputs, fp32 accumulation).  Operand rules as in vw_head_sample; out_logits 16-byte aligned device memory.
 */
vw_status vw_head_logits(vw_handle* handle, const void* hidden, int64_t hidden_stride, int32_t hidden_size,
                         const void* weight, int64_t weight_stride, int32_t n_rows, int32_t vocab, float* out_logits,
                         void* stream);

/*
 * The vocabulary head and the sampler in one call: logits = hidden x weight^T (TalkerModel.CodecHead,
 * TalkerModel.cs:133, or CodePredictorHead, :136-137) on the tcgen05 tensor cores (bf16 inputs, fp32 accumulation and
 * output), then vw_sample over those logits, stream-ordered (the sampler reads the logits while they are in L2).
 * hidden: [segment->n_rows, hidden_size] bf16 (row pitch hidden_stride elements); weight: [segment->vocab,
 * hidden_size] bf16 (pitch weight_stride); both device memory, 16-byte aligned, sizes and pitches multiples of 8.
 * segment: the rows as in vw_sample (histories, steps, mask, opt_index, uniforms, out_ids, out_probs); its logits,
 *   row_stride and dtype are ignored.  vocab must be a multiple of 4.
 * out_logits: optional [n_rows, vocab] fp32 that receives the GEMM's logits; NULL keeps them in a buffer of the
 *   handle.  The ids equal the reference sampler's on these logits; the logits themselves are a bf16 GEMM's (the
 *   reference's CPU GEMM sums in its own order).  Device memory; stream as in vw_sample.
 */
vw_status vw_head_sample(vw_handle* handle, const void* hidden, int64_t hidden_stride, int32_t hidden_size,
                         const void* weight, int64_t weight_stride, const vw_segment* segment,
                         const vw_options* options, int32_t n_options, float* out_logits, void* stream);

/*
 * Single-row mirrors of the reference's Sampler methods, for callers that keep the reference's call shape.
 * Pointers follow `mem`; the calls are synchronous.
 */

/* Sampler.ApplyRepetitionPenalty (Sampler.cs:25-33): in place on `logits[0..vocab)`; each distinct id in
 * `history` is divided (logit >= 0) or multiplied (logit < 0) by `penalty` once. */
vw_status vw_apply_repetition_penalty(vw_handle* handle, float* logits, int32_t vocab, const int32_t* history,
                                      int64_t history_len, float penalty, int32_t mem);

/* Sampler.Select (Sampler.cs:35-88) on one fp32 row, without penalty or mask.  `uniform` is the NextDouble()
 * draw (ignored when options->do_sample == 0).  Unlike the reference, `logits` is not modified. */
vw_status vw_select(vw_handle* handle, const float* logits, int32_t vocab, const vw_options* options,
                    double uniform, int32_t mem, int32_t* out_id);

/* Sampler.ArgMax (Sampler.cs:90-95): first index of the maximum. */
vw_status vw_argmax(vw_handle* handle, const float* logits, int32_t vocab, int32_t mem, int32_t* out_id);

/*
 * Diagnostic: evaluates on the handle's device, for n device doubles x[0..n), the exp the sampler uses for every
 * softmax numerator (exp_libm[i]: glibc's exp restated, so the device reproduces the reference's Math.Exp values,
 * Sampler.cs:57) and CUDA's own exp (exp_cuda[i], for comparison).  Either output may be NULL.  Device memory;
 * synchronous.  No counterpart in the reference: it lets a caller check the device exp against its host libm.
 */
vw_status vw_exp_diagnostic(vw_handle* handle, const double* x, int64_t n, double* exp_libm, double* exp_cuda);

#ifdef __cplusplus
}
#endif

#endif /* VWSAMPLER_H */
