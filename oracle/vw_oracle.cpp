// vw_oracle.cpp -- CPU restatement of voxwerk's token sampler, used as TEST INFRASTRUCTURE ONLY.
//
// Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and `--impl reference` arm) load
// this library, and only as the checker or as the timed CPU baseline.  The shipped sampler
// (voxwerk_b200/csrc) never calls it.
//
// Parity status: UNPINNED.  The reference is managed C# (.NET 10) and cannot be built or run in this
// environment, and its own tests pin only the greedy branch through fixtures that are not distributed with it
// (tests/Voxwerk.Tests/TalkerParityTests.cs:48-106 needs VOXWERK_MODEL_DIR / VOXWERK_REFERENCE_DIR).  Each rule
// below is instead pinned by hand-derived known-answer tests in tests/test_oracle_kat.py.
//
// What is restated, with the precision and order of every operation kept:
//   * Sampler.ApplyRepetitionPenalty      src/Voxwerk/Talker/Sampler.cs:25-33
//   * suppress mask + min_new_tokens      src/Voxwerk/Talker/TalkerGenerator.cs:247-248 (batch form :371-372)
//   * Sampler.Select                      src/Voxwerk/Talker/Sampler.cs:35-88
//   * Sampler.ArgMax                      src/Voxwerk/Talker/Sampler.cs:90-95
//   * bf16 -> fp32 widening (bits << 16)  src/Voxwerk/Numerics/Bf16.cs:13
//   * System.Random(int) NextDouble       .NET BCL (not vendored).  Restated from the published method: Knuth's
//     subtractive generator (TAOCP Vol. 2, 3.2.2) in the Numerical Recipes `ran3` formulation, with the two
//     documented .NET differences (modulus 2^31-1 and a second tap at distance 21 instead of 31).
//
// Mapping of C# semantics to C++:
//   * float arithmetic is IEEE binary32 (SSE), double is binary64; this file is compiled with
//     -ffp-contract=off and without -ffast-math so no multiply-add is fused.
//   * Math.Exp(double) -> std::exp (glibc libm), assumed to be what .NET calls on Linux.
//   * Enumerable.OrderBy is a stable sort -> std::stable_sort.
//   * Enumerable.Sum(IEnumerable<double>) is a sequential index-order loop (assumed: .NET vectorises only the
//     integer overloads).
//   * Array.Sort(float[]) is only used to read the K-th largest value, which any correct selection returns.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

namespace {

struct OracleOptions {           // SamplingOptions (Sampler.cs:4-13) + GenerationOptions.RepetitionPenalty
    int32_t do_sample;           // DoSample
    int32_t top_k;               // TopK
    float top_p;                 // TopP
    float temperature;           // Temperature
    float repetition_penalty;    // GenerationOptions.RepetitionPenalty (TalkerGenerator.cs:11), talker rows only
};

constexpr float kNegInf = -std::numeric_limits<float>::infinity();

inline float bf16_to_float(uint16_t v) {  // Bf16.cs:13
    uint32_t bits = static_cast<uint32_t>(v) << 16;
    float f;
    std::memcpy(&f, &bits, sizeof f);
    return f;
}

// Sampler.ApplyRepetitionPenalty (Sampler.cs:25-33).  Every distinct id is penalised once; an id outside
// [0, n) makes the reference throw (Span indexer), reported here as -1.
int apply_repetition_penalty(float* logits, int n, const int32_t* hist, int64_t hlen, float penalty) {
    if (penalty == 1.0f) return 0;                                   // :27 exact compare
    std::vector<uint8_t> seen(static_cast<size_t>(n), 0);            // history.Distinct() :28
    for (int64_t j = 0; j < hlen; ++j) {
        int32_t id = hist[j];
        if (id < 0 || id >= n) return -1;
        if (seen[id]) continue;
        seen[id] = 1;
        float s = logits[id];                                        // :30
        logits[id] = s < 0 ? s * penalty : s / penalty;              // :31 (fp32 mul / IEEE div)
    }
    return 0;
}

// TalkerGenerator.cs:247-248: ids [lo, hi) except the EOS id are suppressed; EOS as well while t < min_new.
void apply_suppress_mask(float* logits, int n, int lo, int hi, int eos, int step, int min_new) {
    for (int i = std::max(lo, 0); i < std::min(hi, n); ++i)
        if (i != eos) logits[i] = kNegInf;
    if (step < min_new && eos >= 0 && eos < n) logits[eos] = kNegInf;
}

// Sampler.ArgMax (Sampler.cs:90-95): first index of the maximum (strict >).
int argmax(const float* x, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

// Sampler.Select (Sampler.cs:35-88).  `r` is the NextDouble() draw the reference takes at :77; greedy rows
// take no draw.  `probs_out` (nullable, n doubles) receives the final probabilities the draw scans; `exp_args`
// (nullable) collects every argument the softmax passes to Math.Exp (the fp32 difference x - max, :57).
int select(float* logits, int n, const OracleOptions& o, double r, double* probs_out,
           std::vector<float>* exp_args = nullptr) {
    if (!o.do_sample) {                                              // :37
        if (probs_out) std::fill(probs_out, probs_out + n, 0.0);
        return argmax(logits, n);
    }
    const float invT = 1.0f / o.temperature;                         // :39 fp32 division
    for (int i = 0; i < n; ++i) logits[i] *= invT;                   // :40 fp32 multiply

    if (o.top_k > 0 && o.top_k < n) {                                // :42
        std::vector<float> sorted(logits, logits + n);               // :45
        std::nth_element(sorted.begin(), sorted.begin() + (n - o.top_k), sorted.end());
        const float kth = sorted[n - o.top_k];                       // :47 sorted ascending, index n-K
        for (int i = 0; i < n; ++i)
            if (logits[i] < kth) logits[i] = kNegInf;                // :48
    }

    float mx = kNegInf;                                              // :51-52
    for (int i = 0; i < n; ++i) mx = std::max(mx, logits[i]);
    std::vector<double> probs(static_cast<size_t>(n));               // :53
    double sum = 0;
    for (int i = 0; i < n; ++i) {                                    // :55-59
        const float d = logits[i] - mx;                              // fp32 subtraction, then widened
        const bool dropped = std::isinf(logits[i]) && logits[i] < 0;
        probs[i] = dropped ? 0.0 : std::exp(static_cast<double>(d));
        if (exp_args && !dropped) exp_args->push_back(d);
        sum += probs[i];
    }
    for (int i = 0; i < n; ++i) probs[i] /= sum;                     // :60

    if (o.top_p < 1.0f) {                                            // :62
        std::vector<int> idx(static_cast<size_t>(n));                // :65 OrderBy(i => probs[i]), stable
        for (int i = 0; i < n; ++i) idx[i] = i;
        std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return probs[a] < probs[b]; });
        const double thr = static_cast<double>(1.0f - o.top_p);     // :70 `1 - TopP` evaluated in fp32
        double cum = 0;
        for (int j = 0; j < n - 1; ++j) {                            // :67-72
            cum += probs[idx[j]];
            if (cum <= thr) probs[idx[j]] = 0;
            else break;
        }
        sum = 0;                                                     // :73 probs.Sum()
        for (int i = 0; i < n; ++i) sum += probs[i];
        for (int i = 0; i < n; ++i) probs[i] /= sum;                 // :74
    }
    if (probs_out) std::copy(probs.begin(), probs.end(), probs_out);

    double acc = 0;                                                  // :78-87 inverse-CDF draw
    int last = 0;
    for (int i = 0; i < n; ++i) {
        if (probs[i] <= 0) continue;
        acc += probs[i];
        last = i;
        if (r < acc) return i;
    }
    return last;
}

// ---- System.Random(int seed) -- subtractive generator (see header) ----
struct DotNetRandom {
    int32_t seed_array[56];
    int inext, inextp;
};

constexpr int32_t kMBig = 2147483647;   // 2^31 - 1
constexpr int32_t kMSeed = 161803398;   // Knuth / Numerical Recipes seed constant

// C# int arithmetic is unchecked: differences wrap modulo 2^32 (seeds above MSEED make table entries negative).
inline int32_t sub_wrap(int32_t a, int32_t b) {
    return static_cast<int32_t>(static_cast<uint32_t>(a) - static_cast<uint32_t>(b));
}

void dotnet_random_init(DotNetRandom* g, int32_t seed) {
    const int32_t subtraction = (seed == std::numeric_limits<int32_t>::min()) ? kMBig : std::abs(seed);
    int32_t mj = sub_wrap(kMSeed, subtraction);
    g->seed_array[55] = mj;
    int32_t mk = 1;
    for (int i = 1; i < 55; ++i) {       // spread the initial values over the table in steps of 21
        const int ii = (21 * i) % 55;
        g->seed_array[ii] = mk;
        mk = sub_wrap(mj, mk);
        if (mk < 0) mk += kMBig;
        mj = g->seed_array[ii];
    }
    for (int k = 1; k < 5; ++k) {        // four warm-up rounds
        for (int i = 1; i < 56; ++i) {
            int32_t v = sub_wrap(g->seed_array[i], g->seed_array[1 + (i + 30) % 55]);
            if (v < 0) v += kMBig;
            g->seed_array[i] = v;
        }
    }
    g->inext = 0;
    g->inextp = 21;
}

int32_t dotnet_random_sample(DotNetRandom* g) {
    if (++g->inext >= 56) g->inext = 1;
    if (++g->inextp >= 56) g->inextp = 1;
    int32_t v = sub_wrap(g->seed_array[g->inext], g->seed_array[g->inextp]);
    if (v == kMBig) --v;
    if (v < 0) v += kMBig;
    g->seed_array[g->inext] = v;
    return v;
}

double dotnet_random_next_double(DotNetRandom* g) { return dotnet_random_sample(g) * (1.0 / kMBig); }

int sample_row_impl(const void* row, int dtype, int n, int kind, const int32_t* hist, int64_t hlen, int step,
                    const OracleOptions* o, double r, int mask_lo, int mask_hi, int eos, int min_new,
                    int32_t* out_id, double* probs_out, std::vector<float>* exp_args) {
    std::vector<float> lg(static_cast<size_t>(n));
    if (dtype == 0) {
        std::memcpy(lg.data(), row, sizeof(float) * n);
    } else {
        const uint16_t* b = static_cast<const uint16_t*>(row);
        for (int i = 0; i < n; ++i) lg[i] = bf16_to_float(b[i]);
    }
    if (kind == 0) {
        if (apply_repetition_penalty(lg.data(), n, hist, hlen, o->repetition_penalty) != 0) return -1;
        apply_suppress_mask(lg.data(), n, mask_lo, mask_hi, eos, step, min_new);
    }
    *out_id = select(lg.data(), n, *o, r, probs_out, exp_args);
    return 0;
}

}  // namespace

extern "C" {

// One row of the batched call.  Mirrors one iteration of TalkerGenerator.GenerateBatch's talker loop
// (kind 0: penalty + mask + Select, :369-373) or sub-talker loop (kind 1: Select only, :420).
int oracle_sample_row(const void* row, int dtype, int n, int kind, const int32_t* hist, int64_t hlen,
                      int step, const OracleOptions* o, double r, int mask_lo, int mask_hi, int eos,
                      int min_new, int32_t* out_id, double* probs_out) {
    return sample_row_impl(row, dtype, n, kind, hist, hlen, step, o, r, mask_lo, mask_hi, eos, min_new, out_id,
                           probs_out, nullptr);
}

// Batched form over n_rows rows of one segment, split across `n_threads` std::threads.
// hist_offsets: [n_rows+1] CSR offsets (nullable: no history); steps / opt_index nullable.
int oracle_sample_rows(const void* logits, int dtype, int64_t row_stride, int n_rows, int n, int kind,
                       const int64_t* hist_offsets, const int32_t* hist_ids, const int32_t* steps,
                       const int32_t* opt_index, const OracleOptions* opts, const double* uniforms,
                       int mask_lo, int mask_hi, int eos, int min_new, int32_t* out_ids, double* probs_out,
                       int n_threads) {
    const size_t esize = dtype == 0 ? 4 : 2;
    if (n_threads < 1) n_threads = 1;
    std::vector<int> status(static_cast<size_t>(n_threads), 0);
    auto work = [&](int t) {
        const int lo = static_cast<int>(static_cast<int64_t>(n_rows) * t / n_threads);
        const int hi = static_cast<int>(static_cast<int64_t>(n_rows) * (t + 1) / n_threads);
        for (int r = lo; r < hi; ++r) {
            const void* row = static_cast<const char*>(logits) + esize * static_cast<size_t>(row_stride) * r;
            const int32_t* h = nullptr;
            int64_t hl = 0;
            if (hist_offsets) {
                h = hist_ids + hist_offsets[r];
                hl = hist_offsets[r + 1] - hist_offsets[r];
            }
            const int st = steps ? steps[r] : min_new;
            const OracleOptions* o = opts + (opt_index ? opt_index[r] : 0);
            double* po = probs_out ? probs_out + static_cast<size_t>(n) * r : nullptr;
            if (oracle_sample_row(row, dtype, n, kind, h, hl, st, o, uniforms ? uniforms[r] : 0.0, mask_lo,
                                  mask_hi, eos, min_new, out_ids + r, po) != 0)
                status[t] = -1;
        }
    };
    if (n_threads == 1) {
        work(0);
    } else {
        std::vector<std::thread> pool;
        for (int t = 0; t < n_threads; ++t) pool.emplace_back(work, t);
        for (auto& th : pool) th.join();
    }
    for (int s : status)
        if (s != 0) return s;
    return 0;
}

// Single-rule entry points for the known-answer tests.
int oracle_apply_repetition_penalty(float* logits, int n, const int32_t* hist, int64_t hlen, float penalty) {
    return apply_repetition_penalty(logits, n, hist, hlen, penalty);
}
int oracle_select(float* logits, int n, const OracleOptions* o, double r, double* probs_out) {
    return select(logits, n, *o, r, probs_out);
}
int oracle_argmax(const float* x, int n) { return argmax(x, n); }

// System.Random(seed): fill `out` with the first `count` NextDouble() values.
void oracle_dotnet_random(int32_t seed, double* out, int count) {
    DotNetRandom g;
    dotnet_random_init(&g, seed);
    for (int i = 0; i < count; ++i) out[i] = dotnet_random_next_double(&g);
}
// Same stream as integers (Random.Next() == InternalSample()).
void oracle_dotnet_random_next(int32_t seed, int32_t* out, int count) {
    DotNetRandom g;
    dotnet_random_init(&g, seed);
    for (int i = 0; i < count; ++i) out[i] = dotnet_random_sample(&g);
}

// Every argument the rows' softmax passes to Math.Exp (Sampler.cs:57), in row order, as the exact fp32 values
// x - max.  Writes at most `cap` values and returns how many there are in total (-1: a history id out of range).
int64_t oracle_exp_args(const void* logits, int dtype, int64_t row_stride, int n_rows, int n, int kind,
                        const int64_t* hist_offsets, const int32_t* hist_ids, const int32_t* steps,
                        const int32_t* opt_index, const OracleOptions* opts, int mask_lo, int mask_hi, int eos,
                        int min_new, float* out, int64_t cap) {
    const size_t esize = dtype == 0 ? 4 : 2;
    std::vector<float> args;
    int64_t total = 0;
    for (int r = 0; r < n_rows; ++r) {
        const void* row = static_cast<const char*>(logits) + esize * static_cast<size_t>(row_stride) * r;
        const int32_t* h = hist_offsets ? hist_ids + hist_offsets[r] : nullptr;
        const int64_t hl = hist_offsets ? hist_offsets[r + 1] - hist_offsets[r] : 0;
        int32_t id = 0;
        args.clear();
        if (sample_row_impl(row, dtype, n, kind, h, hl, steps ? steps[r] : min_new,
                            opts + (opt_index ? opt_index[r] : 0), 0.0, mask_lo, mask_hi, eos, min_new, &id, nullptr,
                            &args) != 0)
            return -1;
        for (float a : args) {
            if (total < cap) out[total] = a;
            ++total;
        }
    }
    return total;
}

// glibc exp over an array (used to measure the device exp against the host libm).
void oracle_exp(const double* x, double* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = std::exp(x[i]);
}

}  // extern "C"
