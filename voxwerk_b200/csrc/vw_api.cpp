// vw_api.cpp -- C ABI of the sampler (include/vwsampler.h): argument checks, device-memory staging for host
// callers, launch planning and error reporting.  No C++ exception crosses the boundary.

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/vwsampler.h"
#include "vw_internal.h"

#define VW_EXPORT extern "C" __attribute__((visibility("default")))

constexpr int kCopyStreams = 3;   // host -> device copies of VW_MEM_HOST calls run on this many copy engines

struct vw_handle {
    int device = -1;
    cudaStream_t stream = nullptr;
    cudaStream_t copy_streams[kCopyStreams] = {};
    cudaEvent_t copy_events[kCopyStreams + 1] = {};   // one per copy stream, and the fork point
    int sm_count = 0;
    unsigned* d_err = nullptr;      // device error word (kErr* bits)
    unsigned* h_err = nullptr;      // pinned mirror
    char* d_scratch = nullptr;      // general-path scratch, one slice per CTA
    size_t scratch_bytes = 0;
    char* d_stage = nullptr;        // VW_MEM_HOST: device copies of the caller's arrays
    char* d_logits = nullptr;       // vw_head_sample: the GEMM's logits when the caller keeps none
    size_t logits_bytes = 0;
    int32_t* d_defer = nullptr;     // four counters + the rows the warp-per-row kernel defers
    size_t defer_cap = 0;
    size_t stage_bytes = 0;
    vw::DevOptions* d_opts = nullptr;
    vw::DevOptions* h_opts = nullptr;   // pinned upload buffer for option tables > kInlineOptions
    size_t opts_cap = 0;
    cudaEvent_t opts_done = nullptr;
    unsigned long long* d_stats = nullptr;   // vw::kNumStats per-path row counters
    unsigned long long* d_guess = nullptr;   // candidate thresholds carried from call to call
    int force_exact = 0;                     // VW_FORCE_EXACT at creation
    int test_stall_row = -1;                 // VW_TEST_STALL_ROW at creation (first vw_sample call only)
    unsigned long long h2d_bytes = 0;        // host -> device input bytes of VW_MEM_HOST calls (vw_stats.h2d_bytes)
    std::vector<vw_batch*> batches;          // live batches created on this handle (released by vw_destroy)
    std::string last_error;
};

namespace {
void orphan_batch(vw_batch* b);   // frees a batch's device memory and detaches it from its handle
}  // namespace

namespace vw {

void fill_row_layout(DevSegment& d) {
    const int vsh = d.dtype == 0 ? 2 : 3, vwe = 1 << vsh;
    const int V = d.vocab;
    d.vsh = vsh;
    d.va = V >> vsh;   // everything is part A unless a suppress span is skipped
    d.c0 = d.va;
    d.vc = 0;
    d.eosv = -1;
    d.spec_a = 1;
    d.spec_b = 0;
    if (d.kind == 0 && d.sup_lo < d.sup_hi) {
        const int la = (d.sup_lo + vwe - 1) >> vsh << vsh;   // the span's aligned interior [la, ha) is never read
        const int ha = d.sup_hi >> vsh << vsh;
        if (la < ha) {
            d.va = la >> vsh;
            d.c0 = ha >> vsh;
            d.vc = (V >> vsh) - d.c0;
            if (d.eos >= la && d.eos < ha) d.eosv = d.eos >> vsh;
        }
        d.spec_a = d.sup_lo >> vsh;           // vectors holding suppressed ids outside the skipped interior
        d.spec_b = (d.sup_hi - 1) >> vsh;
    }
    d.cpl_a = (d.va + 31) / 32;
    d.cpl_c = (d.vc + 31) / 32;
    d.rw_ok = d.bulk_ok && (V & (vwe - 1)) == 0 && d.cpl_a <= 32 && d.cpl_c <= 32;
}

}  // namespace vw

namespace {

// Restores the caller's current device on scope exit.
class DeviceGuard {
  public:
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
        ok_ = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev_ >= 0) cudaSetDevice(prev_);
    }
    bool ok() const { return ok_; }

  private:
    int prev_ = -1;
    bool ok_ = false;
};

vw_status fail(vw_handle* h, vw_status s, const std::string& msg) {
    if (h) h->last_error = msg;
    return s;
}

vw_status cuda_fail(vw_handle* h, cudaError_t e, const char* where) {
    return fail(h, VW_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

constexpr int kDeferHeader = 4;   // counters ahead of the deferred-row list

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Elements of a row that the kernel stages: everything outside the suppressed span plus the 16-byte vector
// holding EOS, in index order.
int staged_elems(const vw_segment& s) {
    const int vw = s.dtype == VW_F32 ? 4 : 8;
    if (s.kind == VW_ROWS_TALKER) {
        const int lo = std::clamp(s.suppress_lo, 0, s.vocab);
        const int hi = std::clamp(s.suppress_hi, 0, s.vocab);
        if (lo < hi) {
            const int la = (lo + vw - 1) / vw * vw;
            const int ha = hi / vw * vw;
            if (la < ha) return la + vw + (s.vocab - ha);
        }
    }
    return s.vocab;
}

vw_status grow(vw_handle* h, char** buf, size_t* cap, size_t need, const char* what) {
    if (need <= *cap) return VW_OK;
    if (*buf) {
        cudaError_t e = cudaStreamSynchronize(h->stream);
        if (e != cudaSuccess) return cuda_fail(h, e, what);
        cudaFree(*buf);
        *buf = nullptr;
        *cap = 0;
    }
    const size_t n = round_up(need + need / 4, 1 << 20);
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(buf), n);
    if (e != cudaSuccess) return cuda_fail(h, e, what);
    *cap = n;
    return VW_OK;
}

// Per-option constants the kernels would otherwise form on every row: both are single IEEE operations, correctly
// rounded on the host as on the device (Sampler.cs:39: invT = 1f / Temperature).
void fill_inline_constants(vw::LaunchParams& p) {
    for (int i = 0; i < p.n_opts && i < vw::kInlineOptions; ++i) {
        p.inl_inv_t[i] = 1.0f / p.inl_opts[i].temperature;
        p.inl_pen_rcp[i] = 1.0 / static_cast<double>(p.inl_opts[i].rep_penalty);
    }
}

vw_status check_options(vw_handle* h, const vw_options* opts, int32_t n_opts, bool* any_sample) {
    *any_sample = false;
    if (n_opts < 1 || !opts) return fail(h, VW_ERR_INVALID_ARG, "options: at least one entry is required");
    for (int i = 0; i < n_opts; ++i) {
        if (opts[i].do_sample) {
            *any_sample = true;
            if (!(opts[i].temperature > 0.0f))
                return fail(h, VW_ERR_INVALID_ARG,
                            "options[" + std::to_string(i) + "]: temperature must be > 0 when do_sample");
        }
    }
    return VW_OK;
}

vw_status check_segment(vw_handle* h, const vw_segment& s, int i, int32_t n_opts, bool any_sample, int mem) {
    const std::string w = "segment " + std::to_string(i) + ": ";
    if (s.n_rows < 0) return fail(h, VW_ERR_INVALID_ARG, w + "n_rows < 0");
    if (s.vocab < 1) return fail(h, VW_ERR_INVALID_ARG, w + "vocab < 1");
    if (s.dtype != VW_F32 && s.dtype != VW_BF16) return fail(h, VW_ERR_INVALID_ARG, w + "unknown dtype");
    if (s.kind != VW_ROWS_TALKER && s.kind != VW_ROWS_SUB) return fail(h, VW_ERR_INVALID_ARG, w + "unknown kind");
    if (s.n_rows == 0) return VW_OK;
    const size_t es = s.dtype == VW_F32 ? 4 : 2;
    if (!s.logits || !aligned(s.logits, es)) return fail(h, VW_ERR_INVALID_ARG, w + "logits NULL or misaligned");
    if (s.row_stride < s.vocab) return fail(h, VW_ERR_INVALID_ARG, w + "row_stride < vocab");
    if (!s.out_ids || !aligned(s.out_ids, 4)) return fail(h, VW_ERR_INVALID_ARG, w + "out_ids NULL or misaligned");
    if (s.out_probs && !aligned(s.out_probs, 8)) return fail(h, VW_ERR_INVALID_ARG, w + "out_probs misaligned");
    if (any_sample && !s.uniforms) return fail(h, VW_ERR_INVALID_ARG, w + "uniforms NULL with sampling options");
    if (s.uniforms && !aligned(s.uniforms, 8)) return fail(h, VW_ERR_INVALID_ARG, w + "uniforms misaligned");
    if (s.opt_index && !aligned(s.opt_index, 4)) return fail(h, VW_ERR_INVALID_ARG, w + "opt_index misaligned");
    if (s.kind == VW_ROWS_TALKER) {
        if (s.hist_offsets && (!aligned(s.hist_offsets, 8) || !s.hist_ids || !aligned(s.hist_ids, 4)))
            return fail(h, VW_ERR_INVALID_ARG, w + "hist_offsets / hist_ids NULL or misaligned");
        if (s.steps && !aligned(s.steps, 4)) return fail(h, VW_ERR_INVALID_ARG, w + "steps misaligned");
    }
    if (staged_elems(s) * es > static_cast<size_t>(vw::kMaxStageLogitBytes))
        return fail(h, VW_ERR_INVALID_ARG, w + "vocab too large for one row stage");
    if (mem == VW_MEM_HOST) {
        if (s.opt_index)
            for (int r = 0; r < s.n_rows; ++r)
                if (s.opt_index[r] < 0 || s.opt_index[r] >= n_opts)
                    return fail(h, VW_ERR_INVALID_ARG, w + "opt_index out of range at row " + std::to_string(r));
        if (s.kind == VW_ROWS_TALKER && s.hist_offsets) {
            if (s.hist_offsets[0] < 0) return fail(h, VW_ERR_INVALID_ARG, w + "hist_offsets[0] < 0");
            for (int r = 0; r < s.n_rows; ++r)
                if (s.hist_offsets[r + 1] < s.hist_offsets[r])
                    return fail(h, VW_ERR_INVALID_ARG, w + "hist_offsets decrease at row " + std::to_string(r));
        }
    }
    return VW_OK;
}

// Copies one host array into the staging buffer at *off (256-byte aligned); returns the device pointer.
template <typename T>
T* stage_copy(vw_handle* h, const T* src, size_t count, size_t* off, cudaStream_t st, cudaError_t* err) {
    if (!src || count == 0) return nullptr;
    *off = round_up(*off, 256);
    T* dst = reinterpret_cast<T*>(h->d_stage + *off);
    *off += count * sizeof(T);
    if (*err == cudaSuccess) *err = cudaMemcpyAsync(dst, src, count * sizeof(T), cudaMemcpyHostToDevice, st);
    h->h2d_bytes += count * sizeof(T);
    return dst;
}

// The copy streams start after the work already on st (fork) and st continues after them (join).
cudaError_t fork_copies(vw_handle* h, cudaStream_t st) {
    cudaError_t e = cudaEventRecord(h->copy_events[kCopyStreams], st);
    for (int i = 0; i < kCopyStreams && e == cudaSuccess; ++i)
        e = cudaStreamWaitEvent(h->copy_streams[i], h->copy_events[kCopyStreams], 0);
    return e;
}
cudaError_t join_copies(vw_handle* h, cudaStream_t st) {
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < kCopyStreams && e == cudaSuccess; ++i) {
        e = cudaEventRecord(h->copy_events[i], h->copy_streams[i]);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, h->copy_events[i], 0);
    }
    return e;
}

// Logit columns [c0, c1) of every row of segment s, copied into the staging area at dst by 2D copies, the rows
// split over the copy streams.
void stage_columns(vw_handle* h, const vw_segment& s, size_t es, unsigned char* dst, int c0, int c1,
                   cudaError_t* err) {
    if (c1 <= c0) return;
    const size_t pitch = static_cast<size_t>(s.row_stride) * es;
    for (int i = 0; i < kCopyStreams && *err == cudaSuccess; ++i) {
        const int r0 = static_cast<int>(static_cast<int64_t>(s.n_rows) * i / kCopyStreams);
        const int r1 = static_cast<int>(static_cast<int64_t>(s.n_rows) * (i + 1) / kCopyStreams);
        if (r1 <= r0) continue;
        *err = cudaMemcpy2DAsync(dst + r0 * pitch + c0 * es, pitch,
                                 static_cast<const unsigned char*>(s.logits) + r0 * pitch + c0 * es, pitch,
                                 static_cast<size_t>(c1 - c0) * es, r1 - r0, cudaMemcpyHostToDevice,
                                 h->copy_streams[i]);
    }
    h->h2d_bytes += static_cast<size_t>(c1 - c0) * es * s.n_rows;
}

// One large host array into the staging area at *off, split over the copy streams; returns the device pointer.
template <typename T>
T* stage_copy_split(vw_handle* h, const T* src, size_t count, size_t* off, cudaError_t* err) {
    if (!src || count == 0) return nullptr;
    *off = round_up(*off, 256);
    T* dst = reinterpret_cast<T*>(h->d_stage + *off);
    *off += count * sizeof(T);
    for (int i = 0; i < kCopyStreams && *err == cudaSuccess; ++i) {
        const size_t a = count * i / kCopyStreams, b = count * (i + 1) / kCopyStreams;
        if (b > a)
            *err = cudaMemcpyAsync(dst + a, src + a, (b - a) * sizeof(T), cudaMemcpyHostToDevice, h->copy_streams[i]);
    }
    h->h2d_bytes += count * sizeof(T);
    return dst;
}

struct HostStaging {
    std::vector<vw_segment> dev;           // device-side view of each segment
    std::vector<std::vector<int64_t>> offsets;   // re-based history offsets
};

// VW_MEM_HOST: copies every input to the device; outputs get device buffers (copied back afterwards).
vw_status stage_host_inputs(vw_handle* h, const vw_segment* segs, int n, cudaStream_t st, HostStaging* hs) {
    hs->dev.assign(segs, segs + n);
    hs->offsets.resize(n);
    size_t need = 0;
    for (int i = 0; i < n; ++i) {
        const vw_segment& s = segs[i];
        if (s.n_rows == 0) continue;
        const size_t es = s.dtype == VW_F32 ? 4 : 2;
        need += round_up((static_cast<size_t>(s.n_rows - 1) * s.row_stride + s.vocab) * es, 256) + 256;
        if (s.kind == VW_ROWS_TALKER && s.hist_offsets) {
            need += round_up(static_cast<size_t>(s.n_rows + 1) * 8, 256) + 256;
            need += round_up(static_cast<size_t>(s.hist_offsets[s.n_rows] - s.hist_offsets[0]) * 4, 256) + 256;
        }
        if (s.kind == VW_ROWS_TALKER && s.steps) need += round_up(static_cast<size_t>(s.n_rows) * 4, 256) + 256;
        if (s.opt_index) need += round_up(static_cast<size_t>(s.n_rows) * 4, 256) + 256;
        if (s.uniforms) need += round_up(static_cast<size_t>(s.n_rows) * 8, 256) + 256;
        need += round_up(static_cast<size_t>(s.n_rows) * 4, 256) + 256;
        if (s.out_probs) need += round_up(static_cast<size_t>(s.n_rows) * s.vocab * 8, 256) + 256;
    }
    vw_status r = grow(h, &h->d_stage, &h->stage_bytes, need, "staging buffer");
    if (r != VW_OK) return r;
    size_t off = 0;
    cudaError_t e = fork_copies(h, st);
    for (int i = 0; i < n; ++i) {
        const vw_segment& s = segs[i];
        vw_segment& d = hs->dev[i];
        if (s.n_rows == 0) continue;
        const size_t es = s.dtype == VW_F32 ? 4 : 2;
        const size_t nel = static_cast<size_t>(s.n_rows - 1) * s.row_stride + s.vocab;
        // The kernels read, of a talker row with a suppress span, only the columns outside the span's 16-byte
        // aligned interior plus the 16-byte vector holding EOS (the rest become -inf unread).  Those columns are
        // copied as [0, lo_al) (extended over the EOS vector when it lies in the first half of the span) and
        // [hi_al, V); every other segment is copied whole.
        int c_lo = s.vocab, c_hi = s.vocab;
        if (s.kind == VW_ROWS_TALKER) {
            const int vw = s.dtype == VW_F32 ? 4 : 8;
            const int lo = std::clamp(s.suppress_lo, 0, s.vocab), hi = std::clamp(s.suppress_hi, 0, s.vocab);
            const int la = (lo + vw - 1) / vw * vw, ha = hi / vw * vw;
            if (lo < hi && la < ha) {
                c_lo = la;
                c_hi = ha;
                if (s.eos_id >= la && s.eos_id < ha) c_lo = (s.eos_id / vw + 1) * vw;   // through the EOS vector
                if (c_lo - la > (ha - la) / 2) c_lo = c_hi = s.vocab;                    // no saving: copy whole
            }
        }
        if (c_lo < c_hi) {
            off = round_up(off, 256);
            unsigned char* dst = reinterpret_cast<unsigned char*>(h->d_stage) + off;
            off += nel * es;
            stage_columns(h, s, es, dst, 0, c_lo, &e);
            stage_columns(h, s, es, dst, c_hi, s.vocab, &e);
            d.logits = dst;
        } else {
            d.logits = stage_copy_split(h, static_cast<const unsigned char*>(s.logits), nel * es, &off, &e);
        }
        if (s.kind == VW_ROWS_TALKER && s.hist_offsets) {
            auto& ofs = hs->offsets[i];
            ofs.resize(static_cast<size_t>(s.n_rows) + 1);
            for (int k = 0; k <= s.n_rows; ++k) ofs[k] = s.hist_offsets[k] - s.hist_offsets[0];
            d.hist_offsets = stage_copy(h, ofs.data(), ofs.size(), &off, st, &e);
            const size_t nh = static_cast<size_t>(s.hist_offsets[s.n_rows] - s.hist_offsets[0]);
            d.hist_ids = nh ? stage_copy_split(h, s.hist_ids + s.hist_offsets[0], nh, &off, &e) : nullptr;
            if (!d.hist_ids) {
                off = round_up(off, 256);
                d.hist_ids = reinterpret_cast<int32_t*>(h->d_stage + off);   // never read: every history empty
            }
        } else {
            d.hist_offsets = nullptr;
            d.hist_ids = nullptr;
        }
        d.steps = (s.kind == VW_ROWS_TALKER) ? stage_copy(h, s.steps, s.steps ? s.n_rows : 0, &off, st, &e) : nullptr;
        d.opt_index = stage_copy(h, s.opt_index, s.opt_index ? s.n_rows : 0, &off, st, &e);
        d.uniforms = stage_copy(h, s.uniforms, s.uniforms ? s.n_rows : 0, &off, st, &e);
        off = round_up(off, 256);
        d.out_ids = reinterpret_cast<int32_t*>(h->d_stage + off);
        off += static_cast<size_t>(s.n_rows) * 4;
        if (s.out_probs) {
            off = round_up(off, 256);
            d.out_probs = reinterpret_cast<double*>(h->d_stage + off);
            off += static_cast<size_t>(s.n_rows) * s.vocab * 8;
        }
    }
    if (e == cudaSuccess) e = join_copies(h, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "host-to-device copy");
    return VW_OK;
}

vw_status read_device_error(vw_handle* h, cudaStream_t st) {
    cudaError_t e = cudaMemcpyAsync(h->h_err, h->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(h, e, "synchronize");
    const unsigned bits = *h->h_err;
    if (bits) {
        cudaMemsetAsync(h->d_err, 0, sizeof(unsigned), st);
        if (h->d_defer) cudaMemsetAsync(h->d_defer, 0, kDeferHeader * sizeof(int32_t), st);
        cudaStreamSynchronize(st);
    }
    if (bits & vw::kErrTimeout) return fail(h, VW_ERR_TIMEOUT, "a bounded wait in the sampler kernel gave up");
    if (bits & vw::kErrHistRange) return fail(h, VW_ERR_OUT_OF_RANGE, "a history id is outside [0, vocab)");
    if (bits & vw::kErrBadOption) return fail(h, VW_ERR_INVALID_ARG, "a row's opt_index is outside the options table");
    if (bits & vw::kErrHistOffsets) return fail(h, VW_ERR_INVALID_ARG, "hist_offsets are negative or decrease");
    if (bits & vw::kErrCodeRange) return fail(h, VW_ERR_OUT_OF_RANGE, "a frame code is outside its codebook");
    return VW_OK;
}

// Layout of a device-resident batch's rows that vw_segment cannot express (see vw::DevSegment).
struct SegExtra {
    const int32_t* hist_lens;
    int64_t hist_stride;
    const int32_t* active;
};

vw_status sample_impl(vw_handle* h, const vw_segment* segs, int32_t n_segs, const vw_options* opts, int32_t n_opts,
                      int32_t mem, void* stream, const SegExtra* extra = nullptr) {
    if (!h) return VW_ERR_INVALID_ARG;
    h->last_error.clear();
    if (!segs || n_segs < 1 || n_segs > vw::kMaxSegments)
        return fail(h, VW_ERR_INVALID_ARG, "n_segments must be in [1, VW_MAX_SEGMENTS]");
    if (mem != VW_MEM_DEVICE && mem != VW_MEM_HOST) return fail(h, VW_ERR_INVALID_ARG, "unknown memory kind");
    if (mem == VW_MEM_HOST && stream) return fail(h, VW_ERR_INVALID_ARG, "VW_MEM_HOST calls take no stream");
    bool any_sample = false;
    vw_status r = check_options(h, opts, n_opts, &any_sample);
    if (r != VW_OK) return r;
    int64_t total = 0;
    for (int i = 0; i < n_segs; ++i) {
        r = check_segment(h, segs[i], i, n_opts, any_sample, mem);
        if (r != VW_OK) return r;
        total += segs[i].n_rows;
    }
    if (total > INT32_MAX) return fail(h, VW_ERR_INVALID_ARG, "more than 2^31 - 1 rows");
    if (total == 0) return VW_OK;

    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    const bool sync = (stream == nullptr);

    HostStaging hs;
    const vw_segment* run = segs;
    if (mem == VW_MEM_HOST) {
        r = stage_host_inputs(h, segs, n_segs, st, &hs);
        if (r != VW_OK) return r;
        run = hs.dev.data();
    }

    vw::LaunchParams p;
    std::memset(&p, 0, sizeof p);
    int row_begin = 0, vmax = 1, logit_bytes = 16, hist_cap = 0;
    bool any_pen = false;
    for (int i = 0; i < n_opts; ++i) any_pen |= opts[i].repetition_penalty != 1.0f;
    int nd = 0;
    for (int i = 0; i < n_segs; ++i) {
        const vw_segment& s = run[i];
        if (s.n_rows == 0) continue;
        vw::DevSegment& d = p.seg[nd++];
        d.logits = s.logits;
        d.hist_offsets = s.kind == VW_ROWS_TALKER ? s.hist_offsets : nullptr;
        d.hist_ids = s.kind == VW_ROWS_TALKER ? s.hist_ids : nullptr;
        d.steps = s.kind == VW_ROWS_TALKER ? s.steps : nullptr;
        d.opt_index = s.opt_index;
        d.uniforms = s.uniforms;
        d.out_ids = s.out_ids;
        d.out_probs = s.out_probs;
        d.row_stride = s.row_stride;
        d.row_begin = row_begin;
        d.n_rows = s.n_rows;
        d.vocab = s.vocab;
        d.dtype = s.dtype;
        d.kind = s.kind;
        d.sup_lo = s.kind == VW_ROWS_TALKER ? std::clamp(s.suppress_lo, 0, s.vocab) : 0;
        d.sup_hi = s.kind == VW_ROWS_TALKER ? std::clamp(s.suppress_hi, 0, s.vocab) : 0;
        if (d.sup_hi < d.sup_lo) d.sup_hi = d.sup_lo;
        d.eos = s.kind == VW_ROWS_TALKER ? s.eos_id : -1;
        d.min_new = s.kind == VW_ROWS_TALKER ? s.min_new_tokens : 0;
        const size_t es = s.dtype == VW_F32 ? 4 : 2;
        d.bulk_ok = aligned(s.logits, 16) && (s.row_stride * es) % 16 == 0 && (s.vocab * es) % 16 == 0;
        d.hist_aligned = d.hist_ids ? aligned(d.hist_ids, 16) : 0;
        if (extra) {
            d.hist_lens = extra[i].hist_lens;
            d.hist_stride = extra[i].hist_stride;
            d.active = extra[i].active;
        }
        vw::fill_row_layout(d);
        row_begin += s.n_rows;
        vmax = std::max(vmax, s.vocab);
        const int vwe = s.dtype == VW_F32 ? 4 : 8;
        logit_bytes = std::max(logit_bytes, (staged_elems(s) + vwe - 1) / vwe * 16);
        if (s.kind == VW_ROWS_TALKER && s.hist_offsets && any_pen) {
            int hint = s.max_hist_len;
            if (hint <= 0 && mem == VW_MEM_HOST) {
                for (int k = 0; k < s.n_rows; ++k)
                    hint = static_cast<int>(std::min<int64_t>(
                        std::max<int64_t>(hint, segs[i].hist_offsets[k + 1] - segs[i].hist_offsets[k]), vw::kMaxHistStage));
            }
            if (hint <= 0) hint = 1024;
            hist_cap = std::max(hist_cap, static_cast<int>(round_up(std::min(hint, vw::kMaxHistStage), 4)));
        }
    }
    p.n_segs = nd;
    p.total_rows = row_begin;
    p.n_opts = n_opts;
    if (n_opts <= vw::kInlineOptions) {
        std::memcpy(p.inl_opts, opts, sizeof(vw_options) * n_opts);
        fill_inline_constants(p);
    } else {
        if (static_cast<size_t>(n_opts) > h->opts_cap) {
            cudaStreamSynchronize(st);
            if (h->d_opts) cudaFree(h->d_opts);
            if (h->h_opts) cudaFreeHost(h->h_opts);
            h->d_opts = nullptr;
            h->h_opts = nullptr;
            h->opts_cap = 0;
            cudaError_t e = cudaMalloc(&h->d_opts, sizeof(vw::DevOptions) * n_opts);
            if (e == cudaSuccess) e = cudaMallocHost(&h->h_opts, sizeof(vw::DevOptions) * n_opts);
            if (e != cudaSuccess) return cuda_fail(h, e, "options table");
            h->opts_cap = n_opts;
        } else {
            cudaEventSynchronize(h->opts_done);   // the previous upload has left the pinned buffer
        }
        std::memcpy(h->h_opts, opts, sizeof(vw_options) * n_opts);
        cudaError_t e = cudaMemcpyAsync(h->d_opts, h->h_opts, sizeof(vw::DevOptions) * n_opts,
                                        cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaEventRecord(h->opts_done, st);
        if (e != cudaSuccess) return cuda_fail(h, e, "options upload");
        p.dev_opts = h->d_opts;
    }
    p.stage_logit_bytes = logit_bytes;
    p.stage_hist_cap = hist_cap;
    p.flag_bytes = static_cast<int32_t>(round_up(static_cast<size_t>(vmax), 16));
    p.vmax = vmax;
    p.err = h->d_err;
    p.stats = h->d_stats;
    p.guess_seed = h->d_guess;
    p.force_exact = h->force_exact;
    p.wait_ns = h->test_stall_row >= 0 ? vw::kTestWaitLimitNs : vw::kWaitLimitNs;
    p.test_stall_row = h->test_stall_row;
    h->test_stall_row = -1;   // one call only

    // When every segment fits the warp-per-row kernel, no option has a penalty below 1 and every sampling option is a
    // small top-k (0 < K <= 64, K < V), rows reach the whole-row kernel only when their candidates overflow, which is
    // rare: one CTA per SM is enough then, and the launch that usually finds nothing to do costs less (config 2:
    // 29.1 -> 28.6 us per call).  A batch whose rows mostly overflow (all ties) runs at a third of the full grid's
    // whole-row throughput.
    bool rare_defer = true;
    int vmin = INT32_MAX;
    for (int i = 0; i < nd; ++i) {
        rare_defer = rare_defer && p.seg[i].rw_ok;
        vmin = std::min(vmin, p.seg[i].vocab);
    }
    for (int i = 0; i < n_opts && rare_defer; ++i)
        rare_defer = opts[i].repetition_penalty >= 1.0f &&
                     (!opts[i].do_sample || (opts[i].top_k > 0 && opts[i].top_k <= vw::kSmallK && opts[i].top_k < vmin));
    vw::LaunchPlan plan;
    if (!vw::plan_launch(p, h->sm_count, rare_defer ? h->sm_count : INT32_MAX, &plan))
        return fail(h, VW_ERR_INVALID_ARG, "rows too large for shared memory");
    const int grid_g = plan.grid_general;
    p.gscratch_stride = vw::sampler_gscratch_stride(vmax);
    r = grow(h, &h->d_scratch, &h->scratch_bytes, static_cast<size_t>(grid_g) * p.gscratch_stride, "scratch");
    if (r != VW_OK) return r;
    p.gscratch = h->d_scratch;
    // deferred-row list: total_rows entries after four counters (deferred rows, whole-row CTAs done, two spare),
    // all zero between calls
    if (static_cast<size_t>(p.total_rows) + kDeferHeader > h->defer_cap) {
        cudaError_t e = cudaStreamSynchronize(st);
        if (e == cudaSuccess && h->d_defer) e = cudaFree(h->d_defer);
        h->d_defer = nullptr;
        h->defer_cap = 0;
        const size_t cap = static_cast<size_t>(p.total_rows) + kDeferHeader + 4096;
        if (e == cudaSuccess) e = cudaMalloc(&h->d_defer, cap * sizeof(int32_t));
        if (e == cudaSuccess) e = cudaMemset(h->d_defer, 0, kDeferHeader * sizeof(int32_t));
        if (e != cudaSuccess) return cuda_fail(h, e, "deferred-row list");
        h->defer_cap = cap;
    }
    p.deferred_count = reinterpret_cast<uint32_t*>(h->d_defer);
    p.done_count = reinterpret_cast<uint32_t*>(h->d_defer) + 1;
    p.deferred_rows = h->d_defer + kDeferHeader;

    cudaError_t e = cudaSuccess;
    if (sync) e = cudaMemsetAsync(h->d_err, 0, sizeof(unsigned), st);
    if (e == cudaSuccess) e = vw::launch_sampler(p, plan, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "sampler launch");
    if (mem == VW_MEM_HOST) {
        for (int i = 0; i < n_segs && e == cudaSuccess; ++i) {
            const vw_segment& s = segs[i];
            if (s.n_rows == 0) continue;
            e = cudaMemcpyAsync(s.out_ids, hs.dev[i].out_ids, static_cast<size_t>(s.n_rows) * 4,
                                cudaMemcpyDeviceToHost, st);
            if (e == cudaSuccess && s.out_probs)
                e = cudaMemcpyAsync(s.out_probs, hs.dev[i].out_probs, static_cast<size_t>(s.n_rows) * s.vocab * 8,
                                    cudaMemcpyDeviceToHost, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "device-to-host copy");
    }
    if (sync) return read_device_error(h, st);
    return VW_OK;
}

}  // namespace

VW_EXPORT const char* vw_version(void) { return "vwsampler 1.0 (sm_100a)"; }

VW_EXPORT const char* vw_status_string(vw_status s) {
    switch (s) {
        case VW_OK: return "ok";
        case VW_ERR_INVALID_ARG: return "invalid argument";
        case VW_ERR_OUT_OF_RANGE: return "history id out of range";
        case VW_ERR_CUDA: return "CUDA error";
        case VW_ERR_TIMEOUT: return "device wait timed out";
        case VW_ERR_NO_DEVICE: return "no usable CUDA device";
    }
    return "unknown status";
}

VW_EXPORT vw_status vw_create(int32_t device, vw_handle** out) {
    if (!out) return VW_ERR_INVALID_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return VW_ERR_NO_DEVICE;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return VW_ERR_NO_DEVICE;
    DeviceGuard guard(device);
    if (!guard.ok()) return VW_ERR_NO_DEVICE;
    vw_handle* h = new (std::nothrow) vw_handle;
    if (!h) return VW_ERR_CUDA;
    h->device = device;
    h->sm_count = prop.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&h->d_err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMallocHost(&h->h_err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(h->d_err, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->opts_done, cudaEventDisableTiming);
    for (int i = 0; i < kCopyStreams && e == cudaSuccess; ++i)
        e = cudaStreamCreateWithFlags(&h->copy_streams[i], cudaStreamNonBlocking);
    for (int i = 0; i <= kCopyStreams && e == cudaSuccess; ++i)
        e = cudaEventCreateWithFlags(&h->copy_events[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMalloc(&h->d_stats, sizeof(unsigned long long) * vw::kNumStats);
    if (e == cudaSuccess) e = cudaMemset(h->d_stats, 0, sizeof(unsigned long long) * vw::kNumStats);
    constexpr size_t kSeedBytes = sizeof(unsigned long long) * vw::kMaxSegments * vw::kSeedSlots;
    if (e == cudaSuccess) e = cudaMalloc(&h->d_guess, kSeedBytes);
    if (e == cudaSuccess)   // option -1 in every slot: no carried threshold yet
        e = cudaMemset(h->d_guess, 0xff, kSeedBytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    const char* fe = std::getenv("VW_FORCE_EXACT");
    h->force_exact = (fe && fe[0] == '1') ? 1 : 0;
    const char* ts = std::getenv("VW_TEST_STALL_ROW");
    if (ts && ts[0]) h->test_stall_row = std::atoi(ts);
    if (e != cudaSuccess) {
        vw_destroy(h);
        return VW_ERR_CUDA;
    }
    *out = h;
    return VW_OK;
}

VW_EXPORT vw_status vw_destroy(vw_handle* h) {
    if (!h) return VW_OK;
    {
        DeviceGuard guard(h->device);
        if (h->stream) cudaStreamSynchronize(h->stream);
        for (vw_batch* b : h->batches) orphan_batch(b);   // the caller still owns (and destroys) the structs
        h->batches.clear();
        if (h->d_scratch) cudaFree(h->d_scratch);
        if (h->d_stage) cudaFree(h->d_stage);
        if (h->d_logits) cudaFree(h->d_logits);
        if (h->d_opts) cudaFree(h->d_opts);
        if (h->h_opts) cudaFreeHost(h->h_opts);
        if (h->d_err) cudaFree(h->d_err);
        if (h->d_stats) cudaFree(h->d_stats);
        if (h->d_guess) cudaFree(h->d_guess);
        if (h->d_defer) cudaFree(h->d_defer);
        if (h->h_err) cudaFreeHost(h->h_err);
        if (h->opts_done) cudaEventDestroy(h->opts_done);
        if (h->stream) cudaStreamDestroy(h->stream);
        for (int i = 0; i < kCopyStreams; ++i)
            if (h->copy_streams[i]) cudaStreamDestroy(h->copy_streams[i]);
        for (int i = 0; i <= kCopyStreams; ++i)
            if (h->copy_events[i]) cudaEventDestroy(h->copy_events[i]);
    }
    delete h;
    return VW_OK;
}

VW_EXPORT const char* vw_last_error(const vw_handle* h) { return h ? h->last_error.c_str() : ""; }

VW_EXPORT vw_status vw_sample(vw_handle* h, const vw_segment* segs, int32_t n_segs, const vw_options* opts,
                              int32_t n_opts, int32_t mem, void* stream) {
    return sample_impl(h, segs, n_segs, opts, n_opts, mem, stream);
}

VW_EXPORT vw_status vw_synchronize(vw_handle* h, void* stream) {
    if (!h) return VW_ERR_INVALID_ARG;
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    return read_device_error(h, stream ? static_cast<cudaStream_t>(stream) : h->stream);
}

VW_EXPORT vw_status vw_get_stats(vw_handle* h, vw_stats* out, int32_t reset) {
    if (!h) return VW_ERR_INVALID_ARG;
    if (!out) return fail(h, VW_ERR_INVALID_ARG, "NULL out");
    static_assert(sizeof(vw_stats) == sizeof(unsigned long long) * vw::kNumStats, "vw_stats layout");
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaError_t e = cudaMemcpy(out, h->d_stats, sizeof(vw_stats), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && reset) e = cudaMemset(h->d_stats, 0, sizeof(vw_stats));
    if (e == cudaSuccess && reset) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(h, e, "vw_get_stats");
    out->h2d_bytes = h->h2d_bytes;   // host-side counter (the device word in that slot is unused)
    if (reset) h->h2d_bytes = 0;
    return VW_OK;
}

// hidden / weight checks shared by vw_head_logits and vw_head_sample
static vw_status check_head_operands(vw_handle* h, const void* hidden, int64_t hidden_stride, int32_t hidden_size,
                                     const void* weight, int64_t weight_stride, int32_t vocab) {
    if (!hidden || !weight || hidden_size < 8 || hidden_size % 8 != 0 || hidden_stride < hidden_size ||
        weight_stride < hidden_size || hidden_stride % 8 != 0 || weight_stride % 8 != 0 || !aligned(hidden, 16) ||
        !aligned(weight, 16))
        return fail(h, VW_ERR_INVALID_ARG,
                    "hidden / weight: 16-byte aligned bf16 rows, hidden_size and strides multiples of 8");
    if (vocab < 4 || vocab % 4 != 0) return fail(h, VW_ERR_INVALID_ARG, "vocab must be a multiple of 4");
    return VW_OK;
}

// ------------------------------------------------------------------------------------- device-resident batches
// One vw_batch per generation loop: TalkerGenerator.GenerateBatch's per-job state (TalkerGenerator.cs:322-455) in
// device memory, one slot per job, so that a step sends only logits and reads only ids.
struct vw_batch {
    vw_handle* h = nullptr;
    vw::BatchDevice d{};
    double* d_uniforms = nullptr;   // [n_slots] the step's draws
    void* mem = nullptr;            // one allocation for every array
    float* d_logits = nullptr;      // head steps: [n_slots, vocab] logits of the batch's own GEMM
    size_t logits_bytes = 0;
    int32_t vocab = 0, sup_lo = 0, sup_hi = 0, min_new = 0;
};

namespace {

void orphan_batch(vw_batch* b) {
    if (b->mem) cudaFree(b->mem);
    if (b->d_logits) cudaFree(b->d_logits);
    b->mem = nullptr;
    b->d_logits = nullptr;
    b->logits_bytes = 0;
    b->h = nullptr;   // every later call on the batch returns VW_ERR_INVALID_ARG
}

// System.Random(int seed)'s initial state: the published subtractive generator (Knuth, TAOCP Vol. 2 3.2.2;
// Numerical Recipes ran3) with .NET's modulus 2^31 - 1, table spread in steps of 21 and four warm-up rounds.  C#
// int arithmetic wraps, hence the unsigned differences.
void dotnet_seed(int32_t seed, vw::DotNetRngState* g) {
    constexpr int32_t kMBig = 2147483647, kMSeed = 161803398;
    auto sub = [](int32_t a, int32_t b) {
        return static_cast<int32_t>(static_cast<uint32_t>(a) - static_cast<uint32_t>(b));
    };
    const int32_t subtraction = seed == INT32_MIN ? kMBig : (seed < 0 ? -seed : seed);
    int32_t mj = sub(kMSeed, subtraction);
    g->seed[0] = 0;
    g->seed[55] = mj;
    int32_t mk = 1;
    for (int i = 1; i < 55; ++i) {
        const int ii = (21 * i) % 55;
        g->seed[ii] = mk;
        mk = sub(mj, mk);
        if (mk < 0) mk += kMBig;
        mj = g->seed[ii];
    }
    for (int k = 1; k < 5; ++k)
        for (int i = 1; i < 56; ++i) {
            int32_t v = sub(g->seed[i], g->seed[1 + (i + 30) % 55]);
            if (v < 0) v += kMBig;
            g->seed[i] = v;
        }
    g->inext = 0;
    g->inextp = 21;
}

vw_status batch_check(vw_batch* b, const vw_options* options, int32_t n_options) {
    if (!b || !b->h) return VW_ERR_INVALID_ARG;
    b->h->last_error.clear();
    if (!options || n_options < 1 || n_options > vw::kInlineOptions)
        return fail(b->h, VW_ERR_INVALID_ARG, "batch steps take 1.." + std::to_string(vw::kInlineOptions) + " options");
    return VW_OK;
}

std::vector<vw::DevOptions> dev_options(const vw_options* options, int32_t n) {
    std::vector<vw::DevOptions> o(static_cast<size_t>(n));
    std::memcpy(o.data(), options, sizeof(vw_options) * n);
    return o;
}

// A talker or sub-talker step: draws, samples every slot (finished ones get id -1), commits talker ids.
vw_status batch_step(vw_batch* b, int which, const void* logits, int64_t row_stride, int32_t vocab, int32_t dtype,
                     const vw_options* options, int32_t n_options, int32_t* out_ids, int32_t* out_done,
                     void* stream, const vw::EmbedOut* emb = nullptr) {
    vw_status r = batch_check(b, options, n_options);
    if (r != VW_OK) return r;
    vw_handle* h = b->h;
    if (!logits || !out_ids) return fail(h, VW_ERR_INVALID_ARG, "logits and out_ids are required");
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    const std::vector<vw::DevOptions> o = dev_options(options, n_options);
    cudaError_t e = vw::launch_batch_draw(b->d, which, o.data(), n_options, b->d_uniforms, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "batch draw");
    vw_segment sg;
    std::memset(&sg, 0, sizeof sg);
    sg.logits = logits;
    sg.row_stride = row_stride;
    sg.n_rows = b->d.n_slots;
    sg.vocab = vocab;
    sg.dtype = dtype;
    sg.kind = which == 0 ? VW_ROWS_TALKER : VW_ROWS_SUB;
    sg.opt_index = which == 0 ? b->d.opt_talker : b->d.opt_sub;
    sg.uniforms = b->d_uniforms;
    sg.out_ids = out_ids;
    SegExtra ex{nullptr, 0, b->d.active};
    if (which == 0) {
        sg.hist_ids = b->d.history;
        sg.steps = b->d.step;
        sg.suppress_lo = b->sup_lo;
        sg.suppress_hi = b->sup_hi;
        sg.eos_id = b->d.eos;
        sg.min_new_tokens = b->min_new;
        sg.max_hist_len = b->d.max_history;
        ex.hist_lens = b->d.hist_len;
        ex.hist_stride = b->d.max_history;
    }
    r = sample_impl(h, &sg, 1, options, n_options, VW_MEM_DEVICE, st, &ex);
    if (r != VW_OK) return r;
    if (which == 0) {
        e = vw::launch_batch_commit(b->d, out_ids, out_done, emb, h->d_err, st);
        if (e != cudaSuccess) return cuda_fail(h, e, "batch commit");
    }
    if (!stream) return read_device_error(h, st);
    return VW_OK;
}

}  // namespace

VW_EXPORT vw_status vw_batch_create(vw_handle* h, int32_t n_slots, int32_t vocab, int32_t max_history,
                                    int32_t eos_id, int32_t min_new_tokens, int32_t suppress_lo, int32_t suppress_hi,
                                    vw_batch** out) {
    if (!h || !out) return VW_ERR_INVALID_ARG;
    *out = nullptr;
    h->last_error.clear();
    if (n_slots < 1 || vocab < 1 || max_history < 1)
        return fail(h, VW_ERR_INVALID_ARG, "n_slots, vocab and max_history must be >= 1");
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    vw_batch* b = new (std::nothrow) vw_batch;
    if (!b) return fail(h, VW_ERR_CUDA, "out of host memory");
    b->h = h;
    b->vocab = vocab;
    b->sup_lo = suppress_lo;
    b->sup_hi = suppress_hi;
    b->min_new = min_new_tokens;
    const size_t n = static_cast<size_t>(n_slots);
    const size_t hist = round_up(n * static_cast<size_t>(max_history) * 4, 256);
    const size_t ints = round_up(n * 4, 256);
    const size_t rng = round_up(n * sizeof(vw::DotNetRngState), 256);
    const size_t codes = round_up(n * vw::kMaxCodeGroups * 4, 256);
    const size_t total = hist + 6 * ints + 2 * rng + round_up(n * 8, 256) + codes;
    cudaError_t e = cudaMalloc(&b->mem, total);
    if (e == cudaSuccess) e = cudaMemset(b->mem, 0, total);
    if (e != cudaSuccess) {
        delete b;
        return cuda_fail(h, e, "batch state");
    }
    char* p = static_cast<char*>(b->mem);
    auto take = [&](size_t bytes) {
        char* q = p;
        p += bytes;
        return q;
    };
    b->d.n_slots = n_slots;
    b->d.max_history = max_history;
    b->d.eos = eos_id;
    b->d.history = reinterpret_cast<int32_t*>(take(hist));
    b->d.hist_len = reinterpret_cast<int32_t*>(take(ints));
    b->d.step = reinterpret_cast<int32_t*>(take(ints));
    b->d.active = reinterpret_cast<int32_t*>(take(ints));
    b->d.max_new = reinterpret_cast<int32_t*>(take(ints));
    b->d.opt_talker = reinterpret_cast<int32_t*>(take(ints));
    b->d.opt_sub = reinterpret_cast<int32_t*>(take(ints));
    b->d.rng_talker = reinterpret_cast<vw::DotNetRngState*>(take(rng));
    b->d.rng_sub = reinterpret_cast<vw::DotNetRngState*>(take(rng));
    b->d_uniforms = reinterpret_cast<double*>(take(round_up(n * 8, 256)));
    b->d.codes = reinterpret_cast<int32_t*>(take(codes));
    e = cudaMemset(b->d.codes, 0xff, n * vw::kMaxCodeGroups * 4);   // every code -1: no frame yet
    if (e != cudaSuccess) {
        cudaFree(b->mem);
        delete b;
        return cuda_fail(h, e, "batch state");
    }
    h->batches.push_back(b);
    *out = b;
    return VW_OK;
}

VW_EXPORT vw_status vw_batch_destroy(vw_batch* b) {
    if (!b) return VW_OK;
    if (b->h) {   // otherwise vw_destroy of its handle has already released the device memory
        vw_handle* h = b->h;
        DeviceGuard guard(h->device);
        cudaStreamSynchronize(h->stream);
        h->batches.erase(std::remove(h->batches.begin(), h->batches.end(), b), h->batches.end());
        orphan_batch(b);
    }
    delete b;
    return VW_OK;
}

VW_EXPORT vw_status vw_batch_start(vw_batch* b, int32_t slot, const vw_slot_config* cfg, const int32_t* history,
                                   int32_t history_len) {
    if (!b || !b->h) return VW_ERR_INVALID_ARG;
    vw_handle* h = b->h;
    h->last_error.clear();
    if (!cfg || slot < 0 || slot >= b->d.n_slots) return fail(h, VW_ERR_INVALID_ARG, "bad slot or config");
    if (history_len < 0 || (history_len > 0 && !history)) return fail(h, VW_ERR_INVALID_ARG, "bad history");
    if (cfg->max_new_tokens < 1) return fail(h, VW_ERR_INVALID_ARG, "max_new_tokens must be >= 1");
    if (static_cast<int64_t>(history_len) + cfg->max_new_tokens > b->d.max_history)
        return fail(h, VW_ERR_INVALID_ARG, "history_len + max_new_tokens exceeds the batch's max_history");
    for (int32_t i = 0; i < history_len; ++i)
        if (history[i] < 0 || history[i] >= b->vocab) return fail(h, VW_ERR_OUT_OF_RANGE, "history id outside [0, vocab)");
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    // Sampler(Seed) and Sampler(Seed + 1) (TalkerGenerator.cs:345-346); an unseeded job takes a host-drawn seed
    // (the reference's unseeded Random is not reproducible either)
    int32_t seed = cfg->seed;
    if (!cfg->seeded) {
        static std::mutex mu;
        static uint64_t x = 0x9e3779b97f4a7c15ull;
        std::lock_guard<std::mutex> lock(mu);
        x ^= static_cast<uint64_t>(std::chrono::high_resolution_clock::now().time_since_epoch().count());
        x = x * 6364136223846793005ull + 1442695040888963407ull;
        seed = static_cast<int32_t>(x >> 33);
    }
    vw::DotNetRngState g[2];
    dotnet_seed(seed, &g[0]);
    dotnet_seed(static_cast<int32_t>(static_cast<uint32_t>(seed) + 1u), &g[1]);
    const int32_t words[6] = {history_len, 0, 1, cfg->max_new_tokens, cfg->talker_option, cfg->sub_option};
    int32_t* dst[6] = {b->d.hist_len, b->d.step, b->d.active, b->d.max_new, b->d.opt_talker, b->d.opt_sub};
    cudaStream_t st = h->stream;
    cudaError_t e = cudaSuccess;
    for (int k = 0; k < 6 && e == cudaSuccess; ++k)
        e = cudaMemcpyAsync(dst[k] + slot, &words[k], 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b->d.rng_talker + slot, &g[0], sizeof g[0], cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b->d.rng_sub + slot, &g[1], sizeof g[1], cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && history_len > 0)
        e = cudaMemcpyAsync(b->d.history + static_cast<int64_t>(slot) * b->d.max_history, history,
                            static_cast<size_t>(history_len) * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(h, e, "vw_batch_start");
    return VW_OK;
}

VW_EXPORT vw_status vw_batch_stop(vw_batch* b, int32_t slot) {
    if (!b || !b->h) return VW_ERR_INVALID_ARG;
    if (slot < 0 || slot >= b->d.n_slots) return fail(b->h, VW_ERR_INVALID_ARG, "bad slot");
    DeviceGuard guard(b->h->device);
    const int32_t zero = 0;
    cudaError_t e = cudaMemcpyAsync(b->d.active + slot, &zero, 4, cudaMemcpyHostToDevice, b->h->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->h->stream);
    if (e != cudaSuccess) return cuda_fail(b->h, e, "vw_batch_stop");
    return VW_OK;
}

VW_EXPORT vw_status vw_batch_talker_step(vw_batch* b, const void* logits, int64_t row_stride, int32_t dtype,
                                         const vw_options* options, int32_t n_options, int32_t* out_ids,
                                         int32_t* out_done, void* stream) {
    return batch_step(b, 0, logits, row_stride, b ? b->vocab : 0, dtype, options, n_options, out_ids, out_done,
                      stream);
}

VW_EXPORT vw_status vw_batch_sub_step(vw_batch* b, const void* logits, int64_t row_stride, int32_t vocab,
                                      int32_t dtype, const vw_options* options, int32_t n_options, int32_t* out_ids,
                                      void* stream) {
    return batch_step(b, 1, logits, row_stride, vocab, dtype, options, n_options, out_ids, nullptr, stream);
}

namespace {

// A caller's vw_embed_out as the kernels take it; false (with the handle's error set) when it is malformed.
bool embed_out(vw_handle* h, const vw_embed_out* in, vw::EmbedOut* out) {
    if (!in->table || !in->out || in->table_rows < 1 || in->hidden < 8 || in->hidden % 8 != 0 ||
        in->out_stride < in->hidden || in->out_stride % 4 != 0 || !aligned(in->table, 16) || !aligned(in->out, 16)) {
        fail(h, VW_ERR_INVALID_ARG, "embed: 16-byte aligned table and out, hidden a multiple of 8, out_stride >= hidden");
        return false;
    }
    *out = vw::EmbedOut{static_cast<const uint16_t*>(in->table), in->table_rows, in->hidden, in->out, in->out_stride};
    return true;
}

// The head GEMM into the batch's logits buffer (all n_slots rows), then a talker (which 0) or sub-talker step over
// those logits; a sub-talker step records its ids as codebook `group` of each slot's frame.
vw_status batch_head_step(vw_batch* b, int which, int group, const void* hidden, int64_t hidden_stride,
                          int32_t hidden_size, const void* weight, int64_t weight_stride, int32_t vocab,
                          const vw_options* options, int32_t n_options, int32_t* out_ids, int32_t* out_done,
                          const vw_embed_out* embed, void* stream) {
    vw_status r = batch_check(b, options, n_options);
    if (r != VW_OK) return r;
    vw_handle* h = b->h;
    r = check_head_operands(h, hidden, hidden_stride, hidden_size, weight, weight_stride, vocab);
    if (r != VW_OK) return r;
    if (!out_ids) return fail(h, VW_ERR_INVALID_ARG, "out_ids is required");
    if (which == 1 && (group < 1 || group >= vw::kMaxCodeGroups))
        return fail(h, VW_ERR_INVALID_ARG, "group must be in [1, 15]");
    vw::EmbedOut emb{};
    if (embed && !embed_out(h, embed, &emb)) return VW_ERR_INVALID_ARG;
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    const size_t need = static_cast<size_t>(b->d.n_slots) * static_cast<size_t>(vocab) * 4;
    if (need > b->logits_bytes) {
        cudaError_t e = cudaStreamSynchronize(st);   // an earlier step may still read the old buffer
        if (e == cudaSuccess && b->d_logits) e = cudaFree(b->d_logits);
        b->d_logits = nullptr;
        b->logits_bytes = 0;
        if (e == cudaSuccess) e = cudaMalloc(&b->d_logits, need);
        if (e != cudaSuccess) return cuda_fail(h, e, "batch logits buffer");
        b->logits_bytes = need;
    }
    cudaError_t e = stream ? cudaSuccess : cudaMemsetAsync(h->d_err, 0, sizeof(unsigned), st);
    if (e == cudaSuccess)
        e = vw::launch_head_gemm(hidden, hidden_stride, weight, weight_stride, b->d.n_slots, vocab, hidden_size,
                                 b->d_logits, vocab, h->d_err, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "head GEMM");
    r = batch_step(b, which, b->d_logits, vocab, vocab, VW_F32, options, n_options, out_ids, out_done, st,
                   embed ? &emb : nullptr);
    if (r != VW_OK) return r;
    if (which == 1) {
        e = vw::launch_batch_record_codes(b->d, out_ids, group, embed ? &emb : nullptr, h->d_err, st);
        if (e != cudaSuccess) return cuda_fail(h, e, "record codes");
    }
    if (!stream) return read_device_error(h, st);
    return VW_OK;
}

}  // namespace

VW_EXPORT vw_status vw_batch_talker_head_step(vw_batch* b, const void* hidden, int64_t hidden_stride,
                                              int32_t hidden_size, const void* weight, int64_t weight_stride,
                                              const vw_options* options, int32_t n_options, int32_t* out_ids,
                                              int32_t* out_done, const vw_embed_out* embed, void* stream) {
    return batch_head_step(b, 0, 0, hidden, hidden_stride, hidden_size, weight, weight_stride, b ? b->vocab : 0,
                           options, n_options, out_ids, out_done, embed, stream);
}

VW_EXPORT vw_status vw_batch_sub_head_step(vw_batch* b, int32_t group, const void* hidden, int64_t hidden_stride,
                                           int32_t hidden_size, const void* weight, int64_t weight_stride,
                                           int32_t vocab, const vw_options* options, int32_t n_options,
                                           int32_t* out_ids, const vw_embed_out* embed, void* stream) {
    return batch_head_step(b, 1, group, hidden, hidden_stride, hidden_size, weight, weight_stride, vocab, options,
                           n_options, out_ids, nullptr, embed, stream);
}

VW_EXPORT vw_status vw_batch_code_embedding(vw_batch* b, int32_t group, const void* table, int32_t table_rows,
                                            int32_t hidden, float* out, int64_t out_stride, void* stream) {
    if (!b || !b->h) return VW_ERR_INVALID_ARG;
    vw_handle* h = b->h;
    h->last_error.clear();
    if (group < 0 || group >= vw::kMaxCodeGroups) return fail(h, VW_ERR_INVALID_ARG, "group must be in [0, 15]");
    const vw_embed_out in{table, table_rows, hidden, out, out_stride};
    vw::EmbedOut emb{};
    if (!embed_out(h, &in, &emb)) return VW_ERR_INVALID_ARG;
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    cudaError_t e = stream ? cudaSuccess : cudaMemsetAsync(h->d_err, 0, sizeof(unsigned), st);
    if (e == cudaSuccess)
        e = vw::launch_batch_code_embedding(b->d, group, emb, h->d_err, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "code embedding");
    if (!stream) return read_device_error(h, st);
    return VW_OK;
}

VW_EXPORT vw_status vw_batch_frame_embedding(vw_batch* b, int32_t hidden, const uint16_t* codec_embedding,
                                             const uint16_t* const* cp_embeddings, int32_t cp_vocab,
                                             const float* text, float* out, void* stream) {
    if (!b || !b->h) return VW_ERR_INVALID_ARG;
    return vw_frame_embedding(b->h, b->d.codes, b->d.n_slots, vw::kMaxCodeGroups, hidden, codec_embedding, b->vocab,
                              cp_embeddings, cp_vocab, text, out, stream);
}

VW_EXPORT vw_status vw_batch_get_codes(vw_batch* b, int32_t* out) {
    if (!b || !b->h) return VW_ERR_INVALID_ARG;
    vw_handle* h = b->h;
    h->last_error.clear();
    if (!out) return fail(h, VW_ERR_INVALID_ARG, "NULL out");
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaError_t e = cudaStreamSynchronize(h->stream);
    if (e == cudaSuccess)
        e = cudaMemcpy(out, b->d.codes, static_cast<size_t>(b->d.n_slots) * vw::kMaxCodeGroups * 4,
                       cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(h, e, "vw_batch_get_codes");
    return VW_OK;
}

VW_EXPORT vw_status vw_batch_query(vw_batch* b, int32_t slot, int32_t* step, int32_t* history_len, int32_t* active) {
    if (!b || !b->h) return VW_ERR_INVALID_ARG;
    if (slot < 0 || slot >= b->d.n_slots) return fail(b->h, VW_ERR_INVALID_ARG, "bad slot");
    DeviceGuard guard(b->h->device);
    int32_t v[3] = {0, 0, 0};
    cudaError_t e = cudaStreamSynchronize(b->h->stream);
    if (e == cudaSuccess) e = cudaMemcpy(&v[0], b->d.step + slot, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&v[1], b->d.hist_len + slot, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&v[2], b->d.active + slot, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(b->h, e, "vw_batch_query");
    if (step) *step = v[0];
    if (history_len) *history_len = v[1];
    if (active) *active = v[2];
    return VW_OK;
}

VW_EXPORT vw_status vw_frame_embedding(vw_handle* h, const int32_t* codes, int32_t n_rows, int32_t n_groups,
                                       int32_t hidden, const uint16_t* codec_embedding, int32_t vocab,
                                       const uint16_t* const* cp_embeddings, int32_t cp_vocab, const float* text,
                                       float* out, void* stream) {
    if (!h) return VW_ERR_INVALID_ARG;
    h->last_error.clear();
    if (n_rows < 0 || n_groups < 1 || n_groups > vw::kMaxCodeGroups)
        return fail(h, VW_ERR_INVALID_ARG, "n_rows >= 0 and 1 <= n_groups <= 16 are required");
    if (hidden < 8 || hidden % 8 != 0) return fail(h, VW_ERR_INVALID_ARG, "hidden must be a positive multiple of 8");
    if (vocab < 1 || (n_groups > 1 && cp_vocab < 1)) return fail(h, VW_ERR_INVALID_ARG, "vocab sizes must be >= 1");
    if (n_rows == 0) return VW_OK;
    const uint16_t* tables[vw::kMaxCodeGroups] = {codec_embedding};
    if (n_groups > 1 && !cp_embeddings) return fail(h, VW_ERR_INVALID_ARG, "cp_embeddings is required");
    for (int g = 1; g < n_groups; ++g) tables[g] = cp_embeddings[g - 1];
    for (int g = 0; g < n_groups; ++g)
        if (!tables[g] || !aligned(tables[g], 16))
            return fail(h, VW_ERR_INVALID_ARG, "embedding tables must be non-NULL and 16-byte aligned");
    if (!codes || !aligned(codes, 4) || !out || !aligned(out, 16) || (text && !aligned(text, 16)))
        return fail(h, VW_ERR_INVALID_ARG, "codes, text and out must be aligned device arrays");
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    cudaError_t e = stream ? cudaSuccess : cudaMemsetAsync(h->d_err, 0, sizeof(unsigned), st);
    if (e == cudaSuccess)
        e = vw::launch_frame_embedding(codes, n_rows, n_groups, hidden, tables, vocab, cp_vocab, text, out, h->d_err,
                                       st);
    if (e != cudaSuccess) return cuda_fail(h, e, "frame embedding");
    if (!stream) return read_device_error(h, st);
    return VW_OK;
}

VW_EXPORT vw_status vw_head_logits(vw_handle* h, const void* hidden, int64_t hidden_stride, int32_t hidden_size,
                                   const void* weight, int64_t weight_stride, int32_t n_rows, int32_t vocab,
                                   float* out_logits, void* stream) {
    if (!h) return VW_ERR_INVALID_ARG;
    h->last_error.clear();
    vw_status r = check_head_operands(h, hidden, hidden_stride, hidden_size, weight, weight_stride, vocab);
    if (r != VW_OK) return r;
    if (n_rows < 0) return fail(h, VW_ERR_INVALID_ARG, "n_rows < 0");
    if (!out_logits || !aligned(out_logits, 16)) return fail(h, VW_ERR_INVALID_ARG, "out_logits: 16-byte aligned");
    if (n_rows == 0) return VW_OK;
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    cudaError_t e = stream ? cudaSuccess : cudaMemsetAsync(h->d_err, 0, sizeof(unsigned), st);
    if (e == cudaSuccess)
        e = vw::launch_head_gemm(hidden, hidden_stride, weight, weight_stride, n_rows, vocab, hidden_size, out_logits,
                                 vocab, h->d_err, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "head GEMM");
    if (!stream) return read_device_error(h, st);
    return VW_OK;
}

VW_EXPORT vw_status vw_head_sample(vw_handle* h, const void* hidden, int64_t hidden_stride, int32_t hidden_size,
                                   const void* weight, int64_t weight_stride, const vw_segment* segment,
                                   const vw_options* options, int32_t n_options, float* out_logits, void* stream) {
    if (!h) return VW_ERR_INVALID_ARG;
    h->last_error.clear();
    if (!segment) return fail(h, VW_ERR_INVALID_ARG, "segment is required");
    vw_segment sg = *segment;
    vw_status r = check_head_operands(h, hidden, hidden_stride, hidden_size, weight, weight_stride, sg.vocab);
    if (r != VW_OK) return r;
    if (sg.n_rows < 0) return fail(h, VW_ERR_INVALID_ARG, "n_rows < 0");
    if (sg.n_rows == 0) return VW_OK;
    if (out_logits && !aligned(out_logits, 16)) return fail(h, VW_ERR_INVALID_ARG, "out_logits misaligned");
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    float* logits = out_logits;
    if (!logits) {
        r = grow(h, &h->d_logits, &h->logits_bytes, static_cast<size_t>(sg.n_rows) * sg.vocab * 4, "logits buffer");
        if (r != VW_OK) return r;
        logits = reinterpret_cast<float*>(h->d_logits);
    }
    cudaError_t e = stream ? cudaSuccess : cudaMemsetAsync(h->d_err, 0, sizeof(unsigned), st);
    if (e == cudaSuccess)
        e = vw::launch_head_gemm(hidden, hidden_stride, weight, weight_stride, sg.n_rows, sg.vocab, hidden_size,
                                 logits, sg.vocab, h->d_err, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "head GEMM");
    sg.logits = logits;
    sg.row_stride = sg.vocab;
    sg.dtype = VW_F32;
    r = sample_impl(h, &sg, 1, options, n_options, VW_MEM_DEVICE, st);
    if (r != VW_OK) return r;
    if (!stream) return read_device_error(h, st);
    return VW_OK;
}

VW_EXPORT vw_status vw_apply_repetition_penalty(vw_handle* h, float* logits, int32_t vocab, const int32_t* history,
                                                int64_t history_len, float penalty, int32_t mem) {
    if (!h) return VW_ERR_INVALID_ARG;
    h->last_error.clear();
    if (!logits || vocab < 1 || history_len < 0 || (history_len > 0 && !history))
        return fail(h, VW_ERR_INVALID_ARG, "bad logits / history arguments");
    if (mem != VW_MEM_DEVICE && mem != VW_MEM_HOST) return fail(h, VW_ERR_INVALID_ARG, "unknown memory kind");
    if (penalty == 1.0f || history_len == 0) return VW_OK;   // Sampler.cs:27
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t st = h->stream;
    float* d_logits = logits;
    const int32_t* d_hist = history;
    cudaError_t e = cudaSuccess;
    if (mem == VW_MEM_HOST) {
        const size_t need = round_up(static_cast<size_t>(vocab) * 4, 256) + static_cast<size_t>(history_len) * 4 + 256;
        vw_status r = grow(h, &h->d_stage, &h->stage_bytes, need, "staging buffer");
        if (r != VW_OK) return r;
        d_logits = reinterpret_cast<float*>(h->d_stage);
        int32_t* dh = reinterpret_cast<int32_t*>(h->d_stage + round_up(static_cast<size_t>(vocab) * 4, 256));
        e = cudaMemcpyAsync(d_logits, logits, static_cast<size_t>(vocab) * 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(dh, history, static_cast<size_t>(history_len) * 4, cudaMemcpyHostToDevice, st);
        d_hist = dh;
    }
    if (e == cudaSuccess) e = cudaMemsetAsync(h->d_err, 0, sizeof(unsigned), st);
    if (e == cudaSuccess) e = vw::launch_apply_penalty(d_logits, vocab, d_hist, history_len, penalty, h->d_err, st);
    if (e == cudaSuccess && mem == VW_MEM_HOST)
        e = cudaMemcpyAsync(logits, d_logits, static_cast<size_t>(vocab) * 4, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "apply_repetition_penalty");
    return read_device_error(h, st);
}

VW_EXPORT vw_status vw_select(vw_handle* h, const float* logits, int32_t vocab, const vw_options* options,
                              double uniform, int32_t mem, int32_t* out_id) {
    if (!h) return VW_ERR_INVALID_ARG;
    if (!out_id || !options) return fail(h, VW_ERR_INVALID_ARG, "NULL out_id / options");
    vw_segment s;
    std::memset(&s, 0, sizeof s);
    s.logits = logits;
    s.row_stride = vocab;
    s.n_rows = 1;
    s.vocab = vocab;
    s.dtype = VW_F32;
    s.kind = VW_ROWS_SUB;
    double u = uniform;
    if (mem == VW_MEM_HOST) {
        s.uniforms = &u;
        s.out_ids = out_id;
        return sample_impl(h, &s, 1, options, 1, mem, nullptr);
    }
    // device logits: the scalar uniform and the id still live on the host
    s.uniforms = nullptr;
    vw_options o = *options;
    double* d_u = nullptr;
    int32_t* d_id = nullptr;
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    vw_status r = grow(h, &h->d_stage, &h->stage_bytes, 512, "staging buffer");
    if (r != VW_OK) return r;
    d_u = reinterpret_cast<double*>(h->d_stage);
    d_id = reinterpret_cast<int32_t*>(h->d_stage + 256);
    cudaError_t e = cudaMemcpyAsync(d_u, &u, sizeof u, cudaMemcpyHostToDevice, h->stream);
    if (e != cudaSuccess) return cuda_fail(h, e, "select");
    s.uniforms = d_u;
    s.out_ids = d_id;
    r = sample_impl(h, &s, 1, &o, 1, VW_MEM_DEVICE, nullptr);
    if (r != VW_OK) return r;
    e = cudaMemcpy(out_id, d_id, sizeof(int32_t), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(h, e, "select");
    return VW_OK;
}

VW_EXPORT vw_status vw_argmax(vw_handle* h, const float* logits, int32_t vocab, int32_t mem, int32_t* out_id) {
    vw_options o;
    o.do_sample = 0;
    o.top_k = 0;
    o.top_p = 1.0f;
    o.temperature = 1.0f;
    o.repetition_penalty = 1.0f;
    return vw_select(h, logits, vocab, &o, 0.0, mem, out_id);
}

VW_EXPORT vw_status vw_exp_diagnostic(vw_handle* h, const double* x, int64_t n, double* exp_libm,
                                      double* exp_cuda) {
    if (!h) return VW_ERR_INVALID_ARG;
    h->last_error.clear();
    if (n < 0 || (n > 0 && !x)) return fail(h, VW_ERR_INVALID_ARG, "bad argument array");
    if (n == 0) return VW_OK;
    DeviceGuard guard(h->device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    cudaError_t e = vw::launch_exp_diagnostic(x, n, exp_libm, exp_cuda, h->sm_count, h->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
    if (e != cudaSuccess) return cuda_fail(h, e, "exp diagnostic");
    return VW_OK;
}

// ------------------------------------------------------------------------------------- vw_sample_static
// vw_sample for callers that must not allocate device memory: no handle, device pointers only, and the kernels'
// scratch (error word, deferred-row list, whole-row slices) in the fixed array of vw_static.cu.
namespace {

constexpr int kStaticMaxDevices = 64;

struct StaticDevice {
    bool ready = false;
    char* scratch = nullptr;   // device address of the array on this device (looked up on every call)
    int sm_count = 0;
};

std::mutex g_static_mutex;
StaticDevice g_static_devices[kStaticMaxDevices];

void copy_message(const vw_handle& h, char* err_msg, int32_t err_msg_len) {
    if (!err_msg || err_msg_len <= 0) return;
    const size_t n = std::min(h.last_error.size(), static_cast<size_t>(err_msg_len - 1));
    std::memcpy(err_msg, h.last_error.data(), n);
    err_msg[n] = '\0';
}

// Set-up of `device` (current): the array's device address, looked up on every call (cheap, allocates nothing, and
// stays right if the context was reset and the module reloaded), and the SM count, cached.
vw_status static_setup(vw_handle* h, int device, StaticDevice* out) {
    std::lock_guard<std::mutex> lock(g_static_mutex);
    StaticDevice& d = g_static_devices[device];
    if (!d.ready) {
        int sms = 0;
        cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess) return cuda_fail(h, e, "cudaDeviceGetAttribute");
        d.sm_count = sms;
        d.ready = true;
    }
    char* ptr = nullptr;
    cudaError_t e = vw::static_scratch_address(&ptr);
    if (e != cudaSuccess) return cuda_fail(h, e, "cudaGetSymbolAddress of the static scratch");
    if (!ptr) return fail(h, VW_ERR_CUDA, "cudaGetSymbolAddress returned NULL");
    d.scratch = ptr;
    *out = d;
    return VW_OK;
}

vw_status sample_static_impl(vw_handle* h, int32_t device, const vw_segment* segs, int32_t n_segs,
                             const vw_options* opts, int32_t n_opts, void* stream) {
    if (!segs || n_segs < 1 || n_segs > vw::kMaxSegments)
        return fail(h, VW_ERR_INVALID_ARG, "n_segments must be in [1, VW_MAX_SEGMENTS]");
    bool any_sample = false;
    vw_status r = check_options(h, opts, n_opts, &any_sample);
    if (r != VW_OK) return r;
    if (n_opts > vw::kInlineOptions)
        return fail(h, VW_ERR_INVALID_ARG, "vw_sample_static takes at most " + std::to_string(vw::kInlineOptions) +
                                               " options (got " + std::to_string(n_opts) + ")");
    int64_t total = 0;
    for (int i = 0; i < n_segs; ++i) {
        r = check_segment(h, segs[i], i, n_opts, any_sample, VW_MEM_DEVICE);
        if (r != VW_OK) return r;
        if (segs[i].n_rows > 0 && segs[i].vocab > vw::kStaticMaxVocab)
            return fail(h, VW_ERR_INVALID_ARG, "segment " + std::to_string(i) + ": vocab " +
                                                   std::to_string(segs[i].vocab) + " exceeds vw_sample_static's maximum " +
                                                   std::to_string(vw::kStaticMaxVocab));
        total += segs[i].n_rows;
    }
    if (total > vw::kStaticMaxRows)
        return fail(h, VW_ERR_INVALID_ARG, std::to_string(total) + " rows exceed vw_sample_static's maximum of " +
                                               std::to_string(vw::kStaticMaxRows) + " rows per call");
    if (total == 0) return VW_OK;

    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess || device < 0 || device >= n_dev || device >= kStaticMaxDevices)
        return fail(h, VW_ERR_NO_DEVICE, "no CUDA device " + std::to_string(device));
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(h, VW_ERR_CUDA, "cudaSetDevice failed");
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess || major != 10)
        return fail(h, VW_ERR_NO_DEVICE, "device " + std::to_string(device) + " is not an sm_100 device");
    StaticDevice sd;
    r = static_setup(h, device, &sd);
    if (r != VW_OK) return r;
    // every array must be device memory of this device (host memory would need staging buffers, and a kernel
    // given a host or foreign pointer would fault instead of returning a status)
    for (int i = 0; i < n_segs; ++i) {
        const vw_segment& sg = segs[i];
        if (sg.n_rows == 0) continue;
        const bool talker = sg.kind == VW_ROWS_TALKER;
        const void* ptrs[8] = {sg.logits, sg.out_ids, sg.out_probs, sg.uniforms, sg.opt_index,
                               talker ? sg.steps : nullptr, talker ? sg.hist_offsets : nullptr,
                               talker && sg.hist_offsets ? sg.hist_ids : nullptr};
        static const char* names[8] = {"logits", "out_ids", "out_probs", "uniforms", "opt_index", "steps",
                                       "hist_offsets", "hist_ids"};
        for (int k = 0; k < 8; ++k) {
            if (!ptrs[k]) continue;
            cudaPointerAttributes a;
            if (cudaPointerGetAttributes(&a, ptrs[k]) != cudaSuccess ||
                (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) || a.device != device) {
                cudaGetLastError();
                return fail(h, VW_ERR_INVALID_ARG, "segment " + std::to_string(i) + ": " + names[k] +
                                                       " must be device memory of device " + std::to_string(device));
            }
        }
    }

    vw::LaunchParams p;
    std::memset(&p, 0, sizeof p);
    int row_begin = 0, vmax = 1, logit_bytes = 16, hist_cap = 0;
    bool any_pen = false;
    for (int i = 0; i < n_opts; ++i) any_pen |= opts[i].repetition_penalty != 1.0f;
    int nd = 0;
    for (int i = 0; i < n_segs; ++i) {
        const vw_segment& s = segs[i];
        if (s.n_rows == 0) continue;
        vw::DevSegment& d = p.seg[nd++];
        const bool talker = s.kind == VW_ROWS_TALKER;
        d.logits = s.logits;
        d.hist_offsets = talker ? s.hist_offsets : nullptr;
        d.hist_ids = talker ? s.hist_ids : nullptr;
        d.steps = talker ? s.steps : nullptr;
        d.opt_index = s.opt_index;
        d.uniforms = s.uniforms;
        d.out_ids = s.out_ids;
        d.out_probs = s.out_probs;
        d.row_stride = s.row_stride;
        d.row_begin = row_begin;
        d.n_rows = s.n_rows;
        d.vocab = s.vocab;
        d.dtype = s.dtype;
        d.kind = s.kind;
        d.sup_lo = talker ? std::clamp(s.suppress_lo, 0, s.vocab) : 0;
        d.sup_hi = talker ? std::clamp(s.suppress_hi, 0, s.vocab) : 0;
        if (d.sup_hi < d.sup_lo) d.sup_hi = d.sup_lo;
        d.eos = talker ? s.eos_id : -1;
        d.min_new = talker ? s.min_new_tokens : 0;
        const size_t es = s.dtype == VW_F32 ? 4 : 2;
        d.bulk_ok = aligned(s.logits, 16) && (s.row_stride * es) % 16 == 0 && (s.vocab * es) % 16 == 0;
        d.hist_aligned = d.hist_ids ? aligned(d.hist_ids, 16) : 0;
        vw::fill_row_layout(d);
        row_begin += s.n_rows;
        vmax = std::max(vmax, s.vocab);
        const int vwe = s.dtype == VW_F32 ? 4 : 8;
        logit_bytes = std::max(logit_bytes, (staged_elems(s) + vwe - 1) / vwe * 16);
        if (talker && s.hist_offsets && any_pen) {
            const int hint = s.max_hist_len > 0 ? s.max_hist_len : 1024;
            hist_cap = std::max(hist_cap, static_cast<int>(round_up(std::min(hint, vw::kMaxHistStage), 4)));
        }
    }
    p.n_segs = nd;
    p.total_rows = row_begin;
    p.n_opts = n_opts;
    std::memcpy(p.inl_opts, opts, sizeof(vw_options) * n_opts);
    fill_inline_constants(p);
    p.stage_logit_bytes = logit_bytes;
    p.stage_hist_cap = hist_cap;
    p.flag_bytes = static_cast<int32_t>(round_up(static_cast<size_t>(vmax), 16));
    p.vmax = vmax;
    p.stats = nullptr;
    p.wait_ns = vw::kWaitLimitNs;
    p.test_stall_row = -1;
    const char* fe = std::getenv("VW_FORCE_EXACT");
    p.force_exact = (fe && fe[0] == '1') ? 1 : 0;

    vw::LaunchPlan plan;
    if (!vw::plan_launch(p, sd.sm_count, vw::kStaticGeneralCtas, &plan))
        return fail(h, VW_ERR_INVALID_ARG, "rows too large for shared memory");
    p.gscratch_stride = vw::sampler_gscratch_stride(vmax);
    if (p.gscratch_stride > vw::kStaticCtaStride)
        return fail(h, VW_ERR_INVALID_ARG, "vocab too large for the static scratch");
    p.err = reinterpret_cast<unsigned*>(sd.scratch);
    p.deferred_count = reinterpret_cast<uint32_t*>(sd.scratch) + 1;
    p.done_count = reinterpret_cast<uint32_t*>(sd.scratch) + 2;
    p.deferred_rows = reinterpret_cast<int32_t*>(sd.scratch + vw::kStaticRowsOffset);
    p.gscratch = sd.scratch + vw::kStaticScratchOffset;
    p.guess_seed = reinterpret_cast<unsigned long long*>(sd.scratch + vw::kStaticGuessOffset);

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the error word and the counters must start at zero (an earlier call that timed out may have left them
    // set)
    cudaError_t e = cudaMemsetAsync(sd.scratch, 0, 8 * sizeof(uint32_t), st);
    if (e == cudaSuccess) e = vw::launch_sampler(p, plan, st);
    if (e != cudaSuccess) return cuda_fail(h, e, "sampler launch");
    unsigned bits = 0;   // pageable host word: the copy completes before cudaMemcpyAsync returns or at the sync
    e = cudaMemcpyAsync(&bits, sd.scratch, sizeof(unsigned), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(h, e, "synchronize");
    if (bits & vw::kErrTimeout) return fail(h, VW_ERR_TIMEOUT, "a bounded wait in the sampler kernel gave up");
    if (bits & vw::kErrHistRange) return fail(h, VW_ERR_OUT_OF_RANGE, "a history id is outside [0, vocab)");
    if (bits & vw::kErrBadOption) return fail(h, VW_ERR_INVALID_ARG, "a row's opt_index is outside the options table");
    if (bits & vw::kErrHistOffsets) return fail(h, VW_ERR_INVALID_ARG, "hist_offsets are negative or decrease");
    return VW_OK;
}

}  // namespace

VW_EXPORT vw_status vw_sample_static(int32_t device, const vw_segment* segments, int32_t n_segments,
                                     const vw_options* options, int32_t n_options, void* stream, char* err_msg,
                                     int32_t err_msg_len) {
    vw_handle h;   // carries the message only; no device state
    if (err_msg && err_msg_len > 0) err_msg[0] = '\0';
    const vw_status r = sample_static_impl(&h, device, segments, n_segments, options, n_options, stream);
    copy_message(h, err_msg, err_msg_len);
    return r;
}
