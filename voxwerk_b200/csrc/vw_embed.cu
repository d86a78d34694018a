// vw_embed.cu -- the next talker input of every sequence after its frame is sampled (include/vwsampler.h,
// vw_frame_embedding).
//
// voxwerk, per active job after the code predictor (src/Voxwerk/Talker/TalkerGenerator.cs:428-439):
//   TalkerModel.FrameEmbedding(frame, st)   (TalkerModel.cs:114-118): st = bf16->fp32 row codes[0] of the talker
//       codec embedding, then for g = 1..15: st[i] += bf16->fp32 row codes[g] of code-predictor embedding g - 1
//       (CodecEmbedding / CodePredictorEmbedding / AddRow, TalkerModel.cs:96-112, :120-130);
//   st[d] += text[off + d]                  (TalkerGenerator.cs:437-438: the next trailing text row, or tts_pad).
// Every addition is one fp32 rounding in that order, so the result is the reference's bit for bit.  One CTA per row,
// 16-byte loads of 8 bf16 per thread and table; HBM-bound (16 embedding rows + the text row in, one row out).

#include <cuda_runtime.h>

#include "vw_internal.h"

namespace vw {
namespace {

struct EmbedTables {
    const uint16_t* table[kMaxCodeGroups];   // [0]: codec embedding [vocab, H]; [g]: code-predictor g [cp_vocab, H]
};

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }          // Bf16.cs:13
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__global__ void __launch_bounds__(128) frame_embedding_kernel(const int32_t* codes, int n_groups, int hidden,
                                                              EmbedTables t, int vocab, int cp_vocab,
                                                              const float* text, float* out, unsigned* err) {
    const int row = blockIdx.x;
    const int32_t* rc = codes + static_cast<int64_t>(row) * n_groups;
    // a sequence without a frame (a finished slot of vw_batch_talker_step: code 0 is -1); its other codes are not
    // looked at
    if (rc[0] == -1) return;
    __shared__ int32_t code[kMaxCodeGroups];
    __shared__ int skip;
    if (threadIdx.x == 0) skip = 0;
    __syncthreads();
    if (threadIdx.x < n_groups) {
        const int c = rc[threadIdx.x];
        code[threadIdx.x] = c;
        const int lim = threadIdx.x == 0 ? vocab : cp_vocab;
        if (static_cast<unsigned>(c) >= static_cast<unsigned>(lim)) {
            atomicOr(err, kErrCodeRange);   // the reference throws ArgumentOutOfRangeException (TalkerModel.cs:99)
            skip = 1;
        }
    }
    __syncthreads();
    if (skip) return;
    float* o = out + static_cast<int64_t>(row) * hidden;
    const float* tx = text ? text + static_cast<int64_t>(row) * hidden : nullptr;
    for (int i0 = threadIdx.x * 8; i0 < hidden; i0 += blockDim.x * 8) {
        float acc[8];
        {
            const uint4 u = *reinterpret_cast<const uint4*>(t.table[0] + static_cast<int64_t>(code[0]) * hidden + i0);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                acc[2 * k] = bf16_lo(w[k]);
                acc[2 * k + 1] = bf16_hi(w[k]);
            }
        }
        for (int g = 1; g < n_groups; ++g) {   // codebooks 1..15 in order, one rounding per add (AddRow)
            const uint4 u = *reinterpret_cast<const uint4*>(t.table[g] + static_cast<int64_t>(code[g]) * hidden + i0);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                acc[2 * k] = __fadd_rn(acc[2 * k], bf16_lo(w[k]));
                acc[2 * k + 1] = __fadd_rn(acc[2 * k + 1], bf16_hi(w[k]));
            }
        }
        if (tx) {   // + the text row (TalkerGenerator.cs:438)
            const float4 a = *reinterpret_cast<const float4*>(tx + i0);
            const float4 b = *reinterpret_cast<const float4*>(tx + i0 + 4);
            const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = __fadd_rn(acc[k], x[k]);
        }
        *reinterpret_cast<float4*>(o + i0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(o + i0 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

}  // namespace

cudaError_t launch_frame_embedding(const int32_t* codes, int n_rows, int n_groups, int hidden,
                                   const uint16_t* const* tables, int vocab, int cp_vocab, const float* text,
                                   float* out, unsigned* err, cudaStream_t stream) {
    EmbedTables t{};
    for (int g = 0; g < n_groups; ++g) t.table[g] = tables[g];
    if (n_rows > 0)
        frame_embedding_kernel<<<n_rows, 128, 0, stream>>>(codes, n_groups, hidden, t, vocab, cp_vocab, text, out, err);
    return cudaGetLastError();
}

}  // namespace vw
