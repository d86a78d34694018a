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
//     last step, or advances its step (:375-380, :440).
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

__global__ void commit_kernel(BatchDevice b, const int32_t* ids, int32_t* out_done) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= b.n_slots) return;
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

cudaError_t launch_batch_commit(const BatchDevice& b, const int32_t* ids, int32_t* out_done, cudaStream_t stream) {
    const int threads = 128, blocks = (b.n_slots + threads - 1) / threads;
    commit_kernel<<<blocks, threads, 0, stream>>>(b, ids, out_done);
    return cudaGetLastError();
}

}  // namespace vw
