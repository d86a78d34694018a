// vw_batch.cu -- device-resident generation state for a batch of sequences (include/vwsampler.h, vw_batch_*).
//
// voxwerk's TalkerGenerator.GenerateBatch (src/Voxwerk/Talker/TalkerGenerator.cs:322-455) keeps, per active job,
// the talker's generated ids (Active.History, :304), the step counter (Active.Step), the two samplers
// (Sampler(Seed) and Sampler(Seed + 1), :345-346), and retires a job when its code is EOS or its step reaches
// MaxNewTokens - 1 (:375-380).  Here that state lives on the device, one slot per sequence, so a step sends only
// logits and reads only ids:
//   * draw_kernel: one NextDouble() per active sampling slot from the slot's System.Random state (the draw
//     Sampler.Select takes at Sampler.cs:77; greedy slots draw nothing, as the reference's Select returns first);
//   * the sampler kernels read each slot's history in place (row r = slot r);
//   * commit_kernel: appends the talker id to the slot's history (:374), then retires the slot on EOS or on the
//     last step, or advances its step (:375-380, :440), and records code 0 of the frame the slot goes on with;
//   * record_codes_kernel / code_embedding_kernel: each code-predictor group's codes into the frame (:420), and the
//     embedding row of a group's code, the next code-predictor input (:411, :422).
// System.Random(int) is restated from the published subtractive generator (Knuth, TAOCP Vol. 2 3.2.2; Numerical
// Recipes ran3) with .NET's modulus 2^31 - 1 and second tap 21; its state is seeded on the host (vw_api.cpp).

#include <cuda_runtime.h>

#include "vw_internal.h"

namespace vw {
namespace {

constexpr int32_t kMBig = 2147483647;

// Random.NextDouble() on one state (Sampler.cs:77): InternalSample() / (2^31 - 1).
__device__ double rng_next_double(DotNetRngState& g) {
    int inext = g.inext + 1, inextp = g.inextp + 1;
    if (inext >= 56) inext = 1;
    if (inextp >= 56) inextp = 1;
    int32_t v = static_cast<int32_t>(static_cast<uint32_t>(g.seed[inext]) - static_cast<uint32_t>(g.seed[inextp]));
    if (v == kMBig) --v;
    if (v < 0) v += kMBig;
    g.seed[inext] = v;
    g.inext = inext;
    g.inextp = inextp;
    return v * (1.0 / kMBig);
}

struct OptTable {
    DevOptions o[kInlineOptions];
    int32_t n;
};

__global__ void draw_kernel(BatchDevice b, int which, OptTable t, double* uniforms) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= b.n_slots) return;
    double u = 0.0;
    const int oi = which == 0 ? b.opt_talker[s] : b.opt_sub[s];
    if (b.active[s] && oi >= 0 && oi < t.n && t.o[oi].do_sample)
        u = rng_next_double(which == 0 ? b.rng_talker[s] : b.rng_sub[s]);
    uniforms[s] = u;
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }   // Bf16.cs:13
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// out[s] = bf16 -> fp32 of table row `code` (AddRow with add: false, TalkerModel.cs:120-125): the CTA's threads take 8
// values each per step.  A code outside the table sets kErrCodeRange (ArgumentOutOfRangeException, TalkerModel.cs:102,
// 109) and writes nothing.
__device__ __forceinline__ void gather_row(const EmbedOut& e, int s, int code, unsigned* err) {
    if (static_cast<unsigned>(code) >= static_cast<unsigned>(e.table_rows)) {
        if (threadIdx.x == 0) atomicOr(err, kErrCodeRange);
        return;
    }
    const uint16_t* src = e.table + static_cast<int64_t>(code) * e.hidden;
    float* dst = e.out + static_cast<int64_t>(s) * e.out_stride;
    for (int i0 = threadIdx.x * 8; i0 < e.hidden; i0 += blockDim.x * 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(src + i0);
        *reinterpret_cast<float4*>(dst + i0) = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
        *reinterpret_cast<float4*>(dst + i0 + 4) = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
    }
}

// The talker step's bookkeeping for slot s; returns code 0 of the frame slot s goes on with, or -1.
__device__ __forceinline__ int32_t commit_slot(const BatchDevice& b, int s, const int32_t* ids, int32_t* out_done) {
    int32_t done = 0;
    if (b.active[s]) {
        const int32_t id = ids[s];
        const int32_t len = b.hist_len[s];
        if (len < b.max_history) {   // History.Add(code0), TalkerGenerator.cs:374 (vw_batch_start leaves room)
            b.history[static_cast<int64_t>(s) * b.max_history + len] = id;
            b.hist_len[s] = len + 1;
        }
        if (id == b.eos || b.step[s] >= b.max_new[s] - 1) {   // :375-380
            done = 1;
            b.active[s] = 0;
        } else {
            b.step[s] += 1;   // Active.Step++ once the frame is done (:440)
        }
    }
    if (out_done) out_done[s] = done;
    // f[0] = code0 for the jobs that go on to the code predictor (:382-384)
    const int32_t c0 = (b.active[s] && !done) ? ids[s] : -1;
    b.codes[static_cast<int64_t>(s) * kMaxCodeGroups] = c0;
    return c0;
}

__global__ void commit_kernel(BatchDevice b, const int32_t* ids, int32_t* out_done) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s < b.n_slots) commit_slot(b, s, ids, out_done);
}

// commit_kernel and, for every slot that goes on, its CodecEmbedding(code0) row (TalkerGenerator.cs:411): one CTA
// per slot
__global__ void __launch_bounds__(128) commit_embed_kernel(BatchDevice b, const int32_t* ids, int32_t* out_done,
                                                           EmbedOut e, unsigned* err) {
    const int s = blockIdx.x;
    __shared__ int32_t code;
    if (threadIdx.x == 0) code = commit_slot(b, s, ids, out_done);
    __syncthreads();
    if (code >= 0) gather_row(e, s, code, err);
}

__global__ void record_codes_kernel(BatchDevice b, const int32_t* ids, int group) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s < b.n_slots) b.codes[static_cast<int64_t>(s) * kMaxCodeGroups + group] = ids[s];   // keepFrames[i][g] (:420)
}

// record_codes_kernel and, for every slot whose frame goes on, the CodePredictorEmbedding(group, code) row
// (TalkerGenerator.cs:422): one CTA per slot
__global__ void __launch_bounds__(128) record_embed_kernel(BatchDevice b, const int32_t* ids, int group, EmbedOut e,
                                                           unsigned* err) {
    const int s = blockIdx.x;
    const int64_t base = static_cast<int64_t>(s) * kMaxCodeGroups;
    const int32_t id = ids[s];
    if (threadIdx.x == 0) b.codes[base + group] = id;
    if (b.codes[base] < 0 || id < 0) return;   // the slot is idle or retired at this frame's talker step
    gather_row(e, s, id, err);
}

// the gather alone, from the codes table (one CTA per slot)
__global__ void __launch_bounds__(128) code_embedding_kernel(BatchDevice b, int group, EmbedOut e, unsigned* err) {
    const int s = blockIdx.x;
    const int64_t base = static_cast<int64_t>(s) * kMaxCodeGroups;
    if (b.codes[base] < 0) return;   // the slot is idle or retired at this frame's talker step
    gather_row(e, s, b.codes[base + group], err);
}

}  // namespace

cudaError_t launch_batch_draw(const BatchDevice& b, int which, const DevOptions* opts, int n_opts, double* uniforms,
                              cudaStream_t stream) {
    OptTable t;
    t.n = n_opts < kInlineOptions ? n_opts : kInlineOptions;
    for (int i = 0; i < t.n; ++i) t.o[i] = opts[i];
    const int threads = 128, blocks = (b.n_slots + threads - 1) / threads;
    draw_kernel<<<blocks, threads, 0, stream>>>(b, which, t, uniforms);
    return cudaGetLastError();
}

cudaError_t launch_batch_commit(const BatchDevice& b, const int32_t* ids, int32_t* out_done, const EmbedOut* e,
                                unsigned* err, cudaStream_t stream) {
    if (e) {
        commit_embed_kernel<<<b.n_slots, 128, 0, stream>>>(b, ids, out_done, *e, err);
    } else {
        const int threads = 128, blocks = (b.n_slots + threads - 1) / threads;
        commit_kernel<<<blocks, threads, 0, stream>>>(b, ids, out_done);
    }
    return cudaGetLastError();
}

cudaError_t launch_batch_record_codes(const BatchDevice& b, const int32_t* ids, int group, const EmbedOut* e,
                                      unsigned* err, cudaStream_t stream) {
    if (e) {
        record_embed_kernel<<<b.n_slots, 128, 0, stream>>>(b, ids, group, *e, err);
    } else {
        const int threads = 128, blocks = (b.n_slots + threads - 1) / threads;
        record_codes_kernel<<<blocks, threads, 0, stream>>>(b, ids, group);
    }
    return cudaGetLastError();
}

cudaError_t launch_batch_code_embedding(const BatchDevice& b, int group, const EmbedOut& e, unsigned* err,
                                        cudaStream_t stream) {
    code_embedding_kernel<<<b.n_slots, 128, 0, stream>>>(b, group, e, err);
    return cudaGetLastError();
}

}  // namespace vw
