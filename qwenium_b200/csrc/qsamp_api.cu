// qsamp_api.cu -- the C ABI of include/qsamp.h: context, argument checks,
// soft-cap tables, launches, and the host-side allow-mask helpers.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "qsamp_device.h"

extern "C" cudaError_t qs_launch_rows(const qs::QsLaunch* a, int clusters, int cl, size_t smem, cudaStream_t st);
extern "C" cudaError_t qs_kernel_attrs(size_t smem);
extern "C" cudaError_t qs_kernel_static_smem(size_t* out);
extern "C" cudaError_t qs_max_clusters(int cl, size_t smem, int* out);
extern "C" cudaError_t qs_launch_lut(float* lut, float cap, cudaStream_t st);
extern "C" size_t qs_stream_smem(int V);
extern "C" cudaError_t qs_stream_attrs(size_t smem);
extern "C" cudaError_t qs_stream_occupancy(size_t smem, int* blocks_per_sm);
extern "C" cudaError_t qs_launch_stream(const qs::QsLaunch* a, int grid, size_t smem, cudaStream_t st);
extern "C" size_t qs_merge_smem();
extern "C" cudaError_t qs_launch_verify(const void* logits, int dtype, int V, long long row_stride, int n_rows, int B,
                                        const int32_t* row_off, const int32_t* drafts, int eos, int32_t* out_acc,
                                        int32_t* out_bonus, int32_t* out_has, unsigned long long* parts, int segs,
                                        cudaStream_t st);
extern "C" cudaError_t qs_launch_char_class(const uint16_t* table, int V, int B, const uint32_t* classes,
                                            uint32_t* masks, long long mask_stride, int or_into, int num_sms,
                                            cudaStream_t st);
extern "C" cudaError_t qs_merge_attrs(size_t smem);
extern "C" size_t qs_hist_smem();
extern "C" cudaError_t qs_hist_attrs(size_t smem);
extern "C" cudaError_t qs_launch_hist(const qs::QsLaunch* a, int grid, size_t smem, cudaStream_t st);
extern "C" size_t qs_live_smem();
extern "C" int qs_live_vmax();
extern "C" cudaError_t qs_live_attrs(size_t smem);
extern "C" cudaError_t qs_launch_live(const qs::QsLaunch* a, int grid, size_t smem, cudaStream_t st);
extern "C" cudaError_t qs_launch_merge(const qs::QsLaunch* a, const float* all_vals, const int32_t* all_ids,
                                       int n_ranks, int kc, int grid, size_t smem, cudaStream_t st);

namespace {

constexpr int kMaxRounds = 64;

template <typename T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    cudaError_t ensure(size_t want) {
        if (want <= n) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        cudaError_t e = cudaMalloc((void**)&p, want * sizeof(T));
        if (e == cudaSuccess) n = want;
        return e;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
};

}  // namespace

struct qsamp_ctx {
    int device = 0;
    int num_sms = 0;
    int smem_optin = 0;
    std::string err;
    std::mutex mu;
    DevBuf<qsamp_row_params> params;
    DevBuf<int32_t> hist_len;
    DevBuf<double> u;
    DevBuf<qsamp_row_result> results;
    DevBuf<int32_t> rows;          // row lists: streamed rows, then cluster rows
    std::vector<int32_t> h_rows;
    size_t stream_attr = 0;
    bool merge_attr = false;
    DevBuf<int> status;
    DevBuf<float> luts;
    float lut_caps[qs::MAX_LUT] = {0, 0, 0, 0};
    int lut_next = 0;
    // staging for the host-memory entry point
    DevBuf<unsigned char> h_logits;
    DevBuf<int32_t> h_hist, h_ids, h_top_ids;
    DevBuf<uint32_t> h_masks;
    DevBuf<float> h_top_probs;
    DevBuf<qsamp_row_result> h_results;
    cudaStream_t stream = nullptr;
    cudaStream_t aux = nullptr;    // second stream of a call: the stream kernel beside the cluster kernel
    cudaEvent_t fork = nullptr, join = nullptr;
    // third stream: the live-list kernel beside the cluster kernel (fp32
    // full-vocabulary rows shared through a claim queue, lvq)
    cudaStream_t aux2 = nullptr;
    cudaEvent_t fork2 = nullptr, join2 = nullptr;
    DevBuf<int> lvq;
    bool live_last = false;        // the last call ran the live-list kernel
    // host entry point: logits copied in row chunks on a copy stream, each
    // chunk followed by a ready flag (a 4-byte copy from pinned memory)
    cudaStream_t copy = nullptr;
    cudaEvent_t copy_go = nullptr, copy_done = nullptr;
    DevBuf<int> ready;
    DevBuf<unsigned long long> vparts;  // greedy verification: per-segment argmax keys
    int* pinned_one = nullptr;
    // the device status word of the last asynchronous call, copied here in
    // stream order at the end of the call (qsamp_poll_status reads it)
    int* pinned_status = nullptr;
    // device-side bounds (qsamp_set_limits)
    int max_rounds = kMaxRounds;
    unsigned long long ready_wait_ns = 1000000000ull;
    int drop_ready_from = -1;
    // bf16 full-vocabulary rows take the histogram kernel (off: the cluster
    // kernel serves them; qsamp_set_path)
    bool use_hist = true;
    // fp32 full-vocabulary rows shared with the live-list kernel (0, the
    // default: the cluster kernel serves them alone; 2: tests, every row the
    // live-list kernel takes is returned and served by the second cluster
    // launch)
    int use_live = 0;
    bool live_attr = false;
    size_t attrs_smem = 0;
    // clusters the device can place, per cluster size of plan_for, for each
    // (V, layout) seen: device queries that would otherwise run on every call
    struct ClusterOcc {
        int V;
        bool vcounts;
        size_t max_dyn;
        int mc[10];
    };
    std::vector<ClusterOcc> occ;
    size_t max_dyn = 0;    // largest dynamic shared memory a CTA of the kernel may use
    qsamp_counters ctr = {};
    // optional per-kernel device timing: begin / end events of the stream,
    // cluster and merge kernels of the last call
    bool timing = false;
    cudaEvent_t ev[10] = {};
    bool ev_used[5] = {false, false, false, false, false};
    bool hist_attr = false;
};

namespace {

qsamp_status fail(qsamp_ctx* c, qsamp_status s, const char* fmt, ...) {
    if (c) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        c->err = buf;
    }
    return s;
}

qsamp_status cuda_fail(qsamp_ctx* c, cudaError_t e, const char* what) {
    return fail(c, QSAMP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct Plan {
    int cl, n_s, clusters;
    size_t smem;
};

// Smallest cluster whose slices fit the per-CTA shared-memory limit; for
// small batches, wider clusters while every row still gets its own cluster.
// Kernel slots of the timing events.
enum { T_STREAM = 0, T_ROWS = 1, T_MERGE = 2, T_HIST = 3, T_LIVE = 4 };
void t_begin(qsamp_ctx* c, int k, cudaStream_t st) {
    if (c->timing) cudaEventRecord(c->ev[2 * k], st);
}
void t_end(qsamp_ctx* c, int k, cudaStream_t st) {
    c->ctr.kernel_launches += 1;
    if (c->timing) {
        cudaEventRecord(c->ev[2 * k + 1], st);
        c->ev_used[k] = true;
    }
}

qsamp_status plan_for(qsamp_ctx* c, int B, int V, bool vcounts, Plan& out) {
    if (c->max_dyn == 0) {
        size_t st = 0;
        cudaError_t e = qs_kernel_static_smem(&st);
        if (e != cudaSuccess) return cuda_fail(c, e, "cudaFuncGetAttributes");
        c->max_dyn = (size_t)c->smem_optin - st;
    }
    // (the limit may have been computed by another entry point: the
    // kernel's own attributes are set here, once per context)
    if (c->attrs_smem != c->max_dyn) {
        const cudaError_t e = qs_kernel_attrs(c->max_dyn);
        if (e != cudaSuccess) return cuda_fail(c, e, "cudaFuncSetAttribute");
        c->attrs_smem = c->max_dyn;
    }
    // (a GPC holds two clusters of 9 or 10 CTAs but only one of 12 or 16)
    const int sizes[10] = {1, 2, 4, 5, 6, 8, 9, 10, 12, 16};
    int first = -1;
    for (int i = 0; i < 10; ++i) {
        const int n_s = qs::align_up((V + sizes[i] - 1) / sizes[i], 8);
        if ((size_t)qs::smem_layout(n_s, vcounts).total <= c->max_dyn) {
            first = i;
            break;
        }
    }
    if (first < 0)
        return fail(c, QSAMP_ERR_UNSUPPORTED, "V=%d exceeds the largest vocabulary one 16-CTA cluster holds (%d)", V,
                    16 * (int)((c->max_dyn - (size_t)qs::smem_layout(0, vcounts).total) / 4 / 8 * 8));
    // the clusters of each size the device can place (queried once per
    // (V, layout) and context)
    const int* mcs = nullptr;
    for (const auto& o : c->occ)
        if (o.V == V && o.vcounts == vcounts && o.max_dyn == c->max_dyn) mcs = o.mc;
    if (!mcs) {
        qsamp_ctx::ClusterOcc o;
        o.V = V;
        o.vcounts = vcounts;
        o.max_dyn = c->max_dyn;
        for (int i = 0; i < 10; ++i) {
            o.mc[i] = 0;
            if (i < first) continue;
            const int cl = sizes[i];
            const int n_s = qs::align_up((V + cl - 1) / cl, 8);
            const size_t smem = (size_t)qs::smem_layout(n_s, vcounts).total;
            if (qs_max_clusters(cl, smem, &o.mc[i]) != cudaSuccess) {
                cudaGetLastError();
                o.mc[i] = 0;
            }
        }
        c->occ.push_back(o);
        mcs = c->occ.back().mc;
    }
    // (a size the device reports it cannot place -- no cluster of it fits,
    // whatever the reason -- gives way to the next, smaller slices)
    int pick = -1;
    for (int i = first; i < 10; ++i) {
        const int mc = mcs[i];
        if (mc <= 0) {
            if (pick < 0) continue;
            break;
        }
        if (pick < 0 || mc >= B) pick = i;
        if (mc < B) break;
    }
    if (pick < 0)
        return fail(c, QSAMP_ERR_UNSUPPORTED, "V=%d: the device can place no thread-block cluster of the kernel", V);
    const int cl = sizes[pick];
    out.cl = cl;
    out.n_s = qs::align_up((V + cl - 1) / cl, 8);
    out.smem = (size_t)qs::smem_layout(out.n_s, vcounts).total;
    const int mc = mcs[pick];
    out.clusters = mc < B ? mc : B;
    return QSAMP_OK;
}

// V_total > 0: a vocabulary shard (force_token is a global id, outputs are
// the candidate arrays of qsamp_shard_topk, not the batch's).
qsamp_status validate(qsamp_ctx* c, const qsamp_batch* b, int V_total = 0) {
    if (!b) return fail(c, QSAMP_ERR_INVALID_ARG, "batch: expected non-NULL");
    if (b->B < 0) return fail(c, QSAMP_ERR_INVALID_ARG, "B: expected >= 0, got %d", b->B);
    if (b->B == 0) return QSAMP_OK;
    if (b->V < 1) return fail(c, QSAMP_ERR_INVALID_ARG, "V: expected >= 1, got %d", b->V);
    if (b->row_stride < b->V)
        return fail(c, QSAMP_ERR_INVALID_ARG, "row_stride: expected >= V (%d), got %lld", b->V, (long long)b->row_stride);
    if (!b->logits) return fail(c, QSAMP_ERR_INVALID_ARG, "logits: expected non-NULL");
    if (b->dtype != QSAMP_F32 && b->dtype != QSAMP_BF16)
        return fail(c, QSAMP_ERR_INVALID_ARG, "dtype: expected QSAMP_F32 or QSAMP_BF16, got %d", (int)b->dtype);
    if (!b->params) return fail(c, QSAMP_ERR_INVALID_ARG, "params: expected non-NULL");
    if (V_total == 0 && !b->out_ids && !b->out_results)
        return fail(c, QSAMP_ERR_INVALID_ARG, "out_ids/out_results: expected at least one non-NULL");
    const int vt = V_total > 0 ? V_total : b->V;
    if (b->top_cap < 0 || b->top_cap > qs::KMAX)
        return fail(c, QSAMP_ERR_INVALID_ARG, "top_cap: expected [0,%d], got %d", qs::KMAX, b->top_cap);
    if (b->top_cap > 0 && (!b->out_top_ids || !b->out_top_probs))
        return fail(c, QSAMP_ERR_INVALID_ARG, "out_top_ids/out_top_probs: expected non-NULL when top_cap > 0");
    if (b->hist && b->hist_stride < 1)
        return fail(c, QSAMP_ERR_INVALID_ARG, "hist_stride: expected >= 1 with hist, got %d", b->hist_stride);
    const long long words = (b->V + 31) / 32;
    if (b->masks && b->mask_stride != 0 && b->mask_stride < words)
        return fail(c, QSAMP_ERR_INVALID_ARG, "mask_stride: expected 0 or >= %lld words, got %lld", words,
                    (long long)b->mask_stride);
    for (int r = 0; r < b->B; ++r) {
        const qsamp_row_params& p = b->params[r];
        if (p.flags != 0) return fail(c, QSAMP_ERR_INVALID_ARG, "params[%d].flags: expected 0, got %d", r, p.flags);
        if (std::isnan(p.temperature))
            return fail(c, QSAMP_ERR_INVALID_ARG, "params[%d].temperature: expected a number, got NaN", r);
        if (p.force_token < -1 || p.force_token >= vt)
            return fail(c, QSAMP_ERR_INVALID_ARG, "params[%d].force_token: expected -1 or [0,%d), got %d", r, vt,
                        p.force_token);
        if (b->hist) {
            const int len = b->hist_len ? b->hist_len[r] : b->hist_stride;
            if (len < 0 || len > b->hist_stride)
                return fail(c, QSAMP_ERR_INVALID_ARG, "hist_len[%d]: expected [0,%d], got %d", r, b->hist_stride, len);
            const bool pen = p.repetition_penalty != 1.0f || p.frequency_penalty != 0.0f || p.presence_penalty != 0.0f;
            const unsigned long long lb = (unsigned long long)(long long)p.repetition_lookback;
            const long long w = (long long)(lb < (unsigned long long)len ? lb : (unsigned long long)len);
            if (pen && w > qs::HIST_MAX)
                return fail(c, QSAMP_ERR_UNSUPPORTED, "row %d: penalty window of %lld ids exceeds %d", r, w,
                            qs::HIST_MAX);
        }
        if (b->u) {
            const double uu = b->u[r];
            if (!(uu >= 0.0 && uu < 1.0))
                return fail(c, QSAMP_ERR_INVALID_ARG, "u[%d]: expected [0,1), got %g", r, uu);
        }
    }
    return QSAMP_OK;
}

qsamp_status ensure_luts(qsamp_ctx* c, const qsamp_batch* b, cudaStream_t st) {
    if (b->dtype != QSAMP_BF16) return QSAMP_OK;
    cudaError_t e = c->luts.ensure((size_t)qs::MAX_LUT * 65536);
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(soft-cap tables)");
    for (int r = 0; r < b->B; ++r) {
        const float cap = b->params[r].softcap;
        if (!(cap > 0.0f)) continue;
        bool have = false;
        for (int q = 0; q < qs::MAX_LUT; ++q) have |= c->lut_caps[q] == cap;
        if (have) continue;
        // a slot not used by this batch
        int slot = -1;
        for (int t = 0; t < qs::MAX_LUT && slot < 0; ++t) {
            const int q = (c->lut_next + t) % qs::MAX_LUT;
            bool used = false;
            for (int r2 = 0; r2 < b->B && !used; ++r2) used = c->lut_caps[q] != 0.0f && b->params[r2].softcap == c->lut_caps[q];
            if (!used) slot = q;
        }
        if (slot < 0) continue;  // more than MAX_LUT caps: remaining rows compute tanh per element
        e = qs_launch_lut(c->luts.p + (size_t)slot * 65536, cap, st);
        if (e != cudaSuccess) return cuda_fail(c, e, "soft-cap table launch");
        c->ctr.kernel_launches += 1;
        c->lut_caps[slot] = cap;
        c->lut_next = (slot + 1) % qs::MAX_LUT;
    }
    return QSAMP_OK;
}

// The kernels' status word (first error wins) as a qsamp_status.
qsamp_status status_of(qsamp_ctx* c, int st) {
    switch (st) {
        case qs::DEV_OK: return QSAMP_OK;
        case qs::DEV_TOPK_TOO_LARGE: return fail(c, QSAMP_ERR_DEVICE, "device: top-k above the sorted-candidate limit");
        case qs::DEV_ROUNDS_EXHAUSTED:
            return fail(c, QSAMP_ERR_DEVICE,
                        "device: a full-vocabulary row needed more gather rounds than allowed (max_rounds %d; token -1)",
                        c->max_rounds);
        case qs::DEV_TIMEOUT:
            return fail(c, QSAMP_ERR_DEVICE,
                        "device: a bounded wait ran out (row data did not arrive within %llu ns, or a slice copy did "
                        "not complete; token -1)",
                        c->ready_wait_ns);
        default: return fail(c, QSAMP_ERR_DEVICE, "device: internal status %d", st);
    }
}

qsamp_status read_status(qsamp_ctx* c) {
    int st = 0;
    cudaError_t e = cudaMemcpy(&st, c->status.p, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(c, e, "reading the device status");
    c->pinned_status[0] = st;
    return status_of(c, st);
}

// Stream-ordered copy of the status words for qsamp_poll_status (and of the
// count of rows the histogram kernel handed on, and of the rows the live-list
// kernel returned and served, for the counters).
qsamp_status mirror_status(qsamp_ctx* c, cudaStream_t st) {
    cudaError_t e = cudaMemcpyAsync(c->pinned_status, c->status.p, 5 * sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && c->live_last)
        e = cudaMemcpyAsync(c->pinned_status + 5, c->lvq.p + 2, 2 * sizeof(int), cudaMemcpyDeviceToHost, st);
    return e == cudaSuccess ? QSAMP_OK : cuda_fail(c, e, "copying the device status");
}

}  // namespace

extern "C" {

qsamp_status qsamp_create(int32_t device, qsamp_ctx** out) {
    if (!out) return QSAMP_ERR_INVALID_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return QSAMP_ERR_INVALID_ARG;
    }
    qsamp_ctx* c = new (std::nothrow) qsamp_ctx();
    if (!c) return QSAMP_ERR_NO_MEMORY;
    c->device = device;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
    cudaDeviceGetAttribute(&c->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    // [0] status word, [1] cluster row queue, [2] stream row queue, [3] histogram
    // row queue, [4] rows the histogram kernel hands to the cluster kernel
    cudaError_t e = c->status.ensure(8);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->aux, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->join, cudaEventDisableTiming);
    if (e == cudaSuccess) {
        // the live-list kernel's stream takes freed SMs before the stream kernel's
        int lo = 0, hi = 0;
        e = cudaDeviceGetStreamPriorityRange(&lo, &hi);
        if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&c->aux2, cudaStreamNonBlocking, hi);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->fork2, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->join2, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->copy, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->copy_go, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->copy_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaHostAlloc((void**)&c->pinned_one, sizeof(int), cudaHostAllocDefault);
    if (e == cudaSuccess) *c->pinned_one = 1;
    if (e == cudaSuccess) e = cudaHostAlloc((void**)&c->pinned_status, 8 * sizeof(int), cudaHostAllocDefault);
    if (e == cudaSuccess) std::memset(c->pinned_status, 0, 8 * sizeof(int));
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        qsamp_destroy(c);  // releases whatever was created
        return QSAMP_ERR_CUDA;
    }
    *out = c;
    return QSAMP_OK;
}

void qsamp_destroy(qsamp_ctx* c) {
    if (!c) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    c->params.release();
    c->hist_len.release();
    c->u.release();
    c->results.release();
    c->status.release();
    c->luts.release();
    c->h_logits.release();
    c->h_hist.release();
    c->h_ids.release();
    c->h_top_ids.release();
    c->h_masks.release();
    c->h_top_probs.release();
    c->h_results.release();
    c->rows.release();
    c->lvq.release();
    for (cudaEvent_t ev : c->ev)
        if (ev) cudaEventDestroy(ev);
    c->ready.release();
    c->vparts.release();
    if (c->pinned_one) cudaFreeHost(c->pinned_one);
    if (c->pinned_status) cudaFreeHost(c->pinned_status);
    if (c->copy_go) cudaEventDestroy(c->copy_go);
    if (c->copy_done) cudaEventDestroy(c->copy_done);
    if (c->copy) cudaStreamDestroy(c->copy);
    if (c->fork) cudaEventDestroy(c->fork);
    if (c->join) cudaEventDestroy(c->join);
    if (c->aux) cudaStreamDestroy(c->aux);
    if (c->fork2) cudaEventDestroy(c->fork2);
    if (c->join2) cudaEventDestroy(c->join2);
    if (c->aux2) cudaStreamDestroy(c->aux2);
    if (c->stream) cudaStreamDestroy(c->stream);
    cudaSetDevice(prev);
    delete c;
}

const char* qsamp_last_error(const qsamp_ctx* c) { return c ? c->err.c_str() : "no context"; }

// Uploads the per-row parameters, history lengths and uniforms, prepares the
// bf16 soft-cap tables, clears the status word and row queue, and fills the
// launch fields every selection kernel shares. b has been validated.
static qsamp_status common_setup(qsamp_ctx* c, const qsamp_batch* b, cudaStream_t st, qs::QsLaunch& a) {
    const int B = b->B;
    cudaError_t e;
    qsamp_status s;
    if ((e = c->params.ensure(B)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(params)");
    if ((e = c->results.ensure(B)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(results)");
    if ((e = cudaMemcpyAsync(c->params.p, b->params, sizeof(qsamp_row_params) * B, cudaMemcpyHostToDevice, st)) !=
        cudaSuccess)
        return cuda_fail(c, e, "copying params");
    const int32_t* d_hl = nullptr;
    if (b->hist && b->hist_len) {
        if ((e = c->hist_len.ensure(B)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(hist_len)");
        if ((e = cudaMemcpyAsync(c->hist_len.p, b->hist_len, sizeof(int32_t) * B, cudaMemcpyHostToDevice, st)) !=
            cudaSuccess)
            return cuda_fail(c, e, "copying hist_len");
        d_hl = c->hist_len.p;
    }
    const double* d_u = nullptr;
    if (b->u) {
        if ((e = c->u.ensure(B)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(u)");
        if ((e = cudaMemcpyAsync(c->u.p, b->u, sizeof(double) * B, cudaMemcpyHostToDevice, st)) != cudaSuccess)
            return cuda_fail(c, e, "copying u");
        d_u = c->u.p;
    }
    s = ensure_luts(c, b, st);
    if (s != QSAMP_OK) return s;
    if ((e = cudaMemsetAsync(c->status.p, 0, 5 * sizeof(int), st)) != cudaSuccess) return cuda_fail(c, e, "status reset");

    a = qs::QsLaunch{};
    a.logits = b->logits;
    a.dtype = (int)b->dtype;
    a.B = B;
    a.V = b->V;
    a.row_stride = b->row_stride;
    const size_t esz = b->dtype == QSAMP_BF16 ? 2 : 4;
    a.vec_ok = ((uintptr_t)b->logits % 16 == 0) && ((size_t)b->row_stride * esz % 16 == 0);
    a.params = c->params.p;
    a.hist = b->hist;
    a.hist_stride = b->hist_stride;
    a.hist_len = d_hl;
    a.masks = b->masks;
    a.mask_stride = b->mask_stride;
    a.u = d_u;
    a.philox_offset = b->rng_offset;
    a.luts = c->luts.p;
    for (int q = 0; q < qs::MAX_LUT; ++q) a.lut_caps[q] = c->lut_caps[q];
    a.results = b->out_results ? b->out_results : c->results.p;
    a.out_ids = b->out_ids;
    a.top_ids = b->top_cap > 0 ? b->out_top_ids : nullptr;
    a.top_probs = b->top_cap > 0 ? b->out_top_probs : nullptr;
    a.top_cap = b->top_cap;
    a.status = c->status.p;
    a.row_ctr = c->status.p + 1;
    a.srow_ctr = c->status.p + 2;
    a.max_rounds = c->max_rounds;
    a.ready_wait_ns = c->ready_wait_ns;
    return QSAMP_OK;
}

// ready / ready_rows: rows arrive while the kernels run (see qsamp_sample_host);
// null: every row is resident when the kernels start.
static qsamp_status sample_locked(qsamp_ctx* c, const qsamp_batch* b, cudaStream_t st, const int* ready = nullptr,
                                  int ready_rows = 0) {
    qsamp_status s = validate(c, b);
    if (s != QSAMP_OK || b->B == 0) return s;
    const int B = b->B;
    const size_t esz = b->dtype == QSAMP_BF16 ? 2 : 4;
    cudaError_t e;
    qs::QsLaunch a;
    s = common_setup(c, b, st, a);
    if (s != QSAMP_OK) return s;
    a.ready = ready;
    a.ready_rows = ready_rows;
    for (bool& u : c->ev_used) u = false;
    c->ctr.last_cluster_size = 0;
    c->ctr.last_clusters = 0;

    // Route rows: greedy rows and top-k rows (k <= 1024) with a penalty
    // window of at most 1024 ids stream through one CTA each; bf16 rows with
    // a full-vocabulary top-p (and no forced token, no top list, a window of
    // at most 1024 ids) take the histogram kernel; fp32 rows of that kind
    // are shared between the cluster kernel and the live-list kernel; the
    // rest (large k, long windows, top lists) use the cluster kernel, which
    // also serves any row the histogram or live-list kernel hands on.
    const size_t sn_smem = qs_stream_smem(b->V);
    const bool stream_fits = sn_smem <= c->max_dyn || c->max_dyn == 0;
    const size_t hs_smem = qs_hist_smem();
    const bool hist_fits = b->dtype == QSAMP_BF16 && b->top_cap == 0 && hs_smem <= (size_t)c->smem_optin &&
                           c->use_hist;
    const size_t lv_smem = qs_live_smem();
    const bool live_fits = b->dtype == QSAMP_F32 && b->top_cap == 0 && !ready && c->use_live != 0 &&
                           lv_smem <= (size_t)c->smem_optin && b->V <= qs_live_vmax();
    auto window_of = [&](int r) -> long long {
        const qsamp_row_params& p = b->params[r];
        if (!b->hist) return 0;
        const bool pen = p.repetition_penalty != 1.0f || p.frequency_penalty != 0.0f || p.presence_penalty != 0.0f;
        if (!pen) return 0;
        const int len = b->hist_len ? b->hist_len[r] : b->hist_stride;
        const unsigned long long lb = (unsigned long long)(long long)p.repetition_lookback;
        return (long long)(lb < (unsigned long long)len ? lb : (unsigned long long)len);
    };
    auto kind_of = [&](int r) -> int {  // 0 stream, 1 cluster, 2 histogram, 3 cluster or live-list
        const qsamp_row_params& p = b->params[r];
        const long long w = window_of(r);
        if (stream_fits && (p.temperature <= 0.0f || (p.top_k > 0 && p.top_k < b->V && p.top_k <= qs::KMAX)) &&
            w <= 1024)
            return 0;
        const bool full_top_p = p.temperature > 0.0f && !(p.top_k > 0 && p.top_k < b->V) && p.top_p > 0.0f &&
                                p.top_p < 1.0f && p.force_token < 0 && w <= 1024;
        if (hist_fits && full_top_p) return 2;
        if (live_fits && full_top_p) return 3;
        return 1;
    };
    // the row list: stream rows | cluster rows | slots for rows the histogram
    // kernel hands on | histogram rows | rows shared with the live-list kernel
    c->h_rows.resize((size_t)2 * B);
    int n_stream = 0, n_cluster = 0, n_hist = 0, n_live = 0;
    for (int r = 0; r < B; ++r) {
        const int k = kind_of(r);
        n_stream += k == 0;
        n_cluster += k == 1;
        n_hist += k == 2;
        n_live += k == 3;
    }
    const int off_live = n_stream + n_cluster + 2 * n_hist;
    for (int r = 0, i0 = 0, i1 = n_stream, i2 = n_stream + n_cluster + n_hist, i3 = off_live; r < B; ++r) {
        const int k = kind_of(r);
        if (k == 0) c->h_rows[(size_t)i0++] = r;
        else if (k == 1) c->h_rows[(size_t)i1++] = r;
        else if (k == 2) c->h_rows[(size_t)i2++] = r;
        else c->h_rows[(size_t)i3++] = r;
    }
    // Cluster rows are served from a queue in list order: the ones likely to
    // take longest go first, so that they do not start last and set the
    // kernel's length. A higher temperature flattens the row (more logits
    // within reach of the maximum: heavier passes and walks), a top-p cutoff
    // adds the cumulative walk; the key is the temperature, plus one for a
    // cutoff. When rows arrive in chunks, rows of earlier chunks go first.
    // The rows shared with the live-list kernel are ordered the same way: the
    // cluster kernel takes the flattest from the front, the live-list kernel
    // the most peaked from the back.
    auto by_weight = [&](int x, int y) {
        if (ready_rows > 0 && x / ready_rows != y / ready_rows) return x / ready_rows < y / ready_rows;
        auto key = [&](int r) {
            const qsamp_row_params& p = b->params[r];
            const float T = p.temperature > 0.0f ? p.temperature : 0.0f;
            return T + ((p.top_p > 0.0f && p.top_p < 1.0f) ? 1.0f : 0.0f);
        };
        return key(x) > key(y);
    };
    std::stable_sort(c->h_rows.begin() + n_stream, c->h_rows.begin() + n_stream + n_cluster, by_weight);
    std::stable_sort(c->h_rows.begin() + off_live, c->h_rows.begin() + off_live + n_live, by_weight);
    const int nlist = off_live + n_live;
    if ((e = c->rows.ensure(nlist > 0 ? nlist : 1)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(rows)");
    if ((e = cudaMemcpyAsync(c->rows.p, c->h_rows.data(), sizeof(int32_t) * nlist, cudaMemcpyHostToDevice, st)) !=
        cudaSuccess)
        return cuda_fail(c, e, "copying row lists");
    c->live_last = n_live > 0;
    if (n_live > 0) {
        // the claim queue: [0] front, [1] back, [2] returned, [3] served, then
        // the claim words, the return list and the return claims
        const size_t nq = 4 + 3 * (size_t)n_live;
        if ((e = c->lvq.ensure(nq)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(live-list queue)");
        if ((e = cudaMemsetAsync(c->lvq.p, 0, nq * sizeof(int), st)) != cudaSuccess)
            return cuda_fail(c, e, "live-list queue reset");
        a.lv_rows = c->rows.p + off_live;
        a.lv_n = n_live;
        a.lv_q = c->lvq.p;
        a.lv_taken = c->lvq.p + 4;
        a.lv_ret = c->lvq.p + 4 + n_live;
        a.lv_rclaim = c->lvq.p + 4 + 2 * (size_t)n_live;
        a.lv_serve_returns = c->use_live == 2 ? 0 : 1;
        a.lv_return_all = c->use_live == 2 ? 1 : 0;
    }

    // With stream rows and other rows, the others go first on the caller's
    // stream and the stream kernel runs beside them on the context's second
    // stream; the caller's stream then waits for both (fork / join events).
    // The live-list kernel runs on a third stream beside the cluster kernel;
    // a second cluster launch after both serves the rows it returned that
    // the first did not take.
    const bool both = n_stream > 0 && (n_cluster > 0 || n_hist > 0 || n_live > 0);
    cudaStream_t st2 = both ? c->aux : st;
    if (both) {
        if ((e = cudaEventRecord(c->fork, st)) != cudaSuccess || (e = cudaStreamWaitEvent(st2, c->fork, 0)) != cudaSuccess)
            return cuda_fail(c, e, "fork to the second stream");
    }
    if (n_live > 0) {
        if ((e = cudaEventRecord(c->fork2, st)) != cudaSuccess ||
            (e = cudaStreamWaitEvent(c->aux2, c->fork2, 0)) != cudaSuccess)
            return cuda_fail(c, e, "fork to the third stream");
    }
    if (n_hist > 0) {
        if (!c->hist_attr) {
            if ((e = qs_hist_attrs(hs_smem)) != cudaSuccess) return cuda_fail(c, e, "histogram kernel attributes");
            c->hist_attr = true;
        }
        qs::QsLaunch ha = a;
        ha.hs_rows = c->rows.p + n_stream + n_cluster + n_hist;
        ha.hs_nrows = n_hist;
        ha.hs_ctr = c->status.p + 3;
        ha.bail_rows = c->rows.p + n_stream + n_cluster;
        ha.bail_ctr = c->status.p + 4;
        const int grid = n_hist < c->num_sms ? n_hist : c->num_sms;
        t_begin(c, T_HIST, st);
        if ((e = qs_launch_hist(&ha, grid, hs_smem, st)) != cudaSuccess) return cuda_fail(c, e, "histogram kernel launch");
        t_end(c, T_HIST, st);
    }
    Plan plan;
    int live_grid = 0;
    if (n_cluster > 0 || n_hist > 0 || n_live > 0) {
        s = plan_for(c, n_cluster + n_hist + n_live, b->V, b->dtype == QSAMP_BF16, plan);
        if (s != QSAMP_OK) return s;
        if (n_live > 0) {
            // the live-list kernel's CTAs (one SM each), taken from the stream
            // kernel's share: about 100 SM-us per peaked row, and a flat row
            // costs it two passes before it returns it; 4 to 16 CTAs (config2
            // batches, measured on B200: 4 CTAs best; temperatures 0.2-0.6: 16)
            const double wl = 100.0 * 0.4 * n_live;
            const double wc = 140.0 * (0.55 * plan.cl + 2.7) * (n_cluster + 0.6 * n_live);
            const double ws = 48.0 * n_stream;
            live_grid = (int)std::ceil(c->num_sms * wl / (wl + wc + ws));
            live_grid = std::max(std::min(4, n_live), std::min(std::min(live_grid, 16), n_live));
        }
        if (n_stream > 0 && (n_cluster > 0 || n_live > 0)) {
            // the SMs split by the rows' expected work (measured on B200, V=151936):
            // a stream row takes about 48 SM-us (half an SM for ~95 us), a
            // cluster row about 140 us on each of its 6 CTAs' SMs, of which
            // 0.45 scales with the slice (1 / cl) and 0.55 does not; clusters
            // leave the stream kernel its share (and the live-list kernel its CTAs)
            // (the rows shared with the live-list kernel count as cluster rows:
            // fewer clusters cost more than the live-list kernel saves)
            const double ws = 48.0 * n_stream, wc = 140.0 * (0.55 * plan.cl + 2.7) * (n_cluster + n_live);
            const int reserve = (int)std::ceil(c->num_sms * ws / (ws + wc));
            const int cap = (c->num_sms - reserve) / plan.cl;
            plan.clusters = std::max(1, std::min(plan.clusters, cap));
        }
        if (n_live > 0) {
            // launched first: its CTAs take their SMs before the stream
            // kernel's fill the rest (a CTA of it needs a whole SM)
            if (!c->live_attr) {
                if ((e = qs_live_attrs(lv_smem)) != cudaSuccess) return cuda_fail(c, e, "live-list kernel attributes");
                c->live_attr = true;
            }
            t_begin(c, T_LIVE, c->aux2);
            if ((e = qs_launch_live(&a, live_grid, lv_smem, c->aux2)) != cudaSuccess)
                return cuda_fail(c, e, "live-list kernel launch");
            t_end(c, T_LIVE, c->aux2);
        }
        qs::QsLaunch ca = a;
        ca.rows = c->rows.p + n_stream;
        ca.nrows = n_cluster;
        ca.nrows_dev = n_hist > 0 ? c->status.p + 4 : nullptr;
        ca.n_s = plan.n_s;
        c->ctr.last_cluster_size = plan.cl;
        c->ctr.last_clusters = plan.clusters;
        t_begin(c, T_ROWS, st);
        e = qs_launch_rows(&ca, plan.clusters, plan.cl, plan.smem, st);
        if (e != cudaSuccess) return cuda_fail(c, e, "selection kernel launch");
        t_end(c, T_ROWS, st);
    }
    if (n_stream > 0) {
        if (sn_smem > c->stream_attr) {
            if ((e = qs_stream_attrs(sn_smem)) != cudaSuccess) return cuda_fail(c, e, "stream kernel attributes");
            c->stream_attr = sn_smem;
        }
        int per_sm = 0;
        if ((e = qs_stream_occupancy(sn_smem, &per_sm)) != cudaSuccess || per_sm <= 0)
            return cuda_fail(c, e == cudaSuccess ? cudaErrorInvalidConfiguration : e, "stream kernel occupancy");
        qs::QsLaunch sa = a;
        sa.rows = c->rows.p;
        sa.nrows = n_stream;
        const int grid = n_stream < per_sm * c->num_sms ? n_stream : per_sm * c->num_sms;
        t_begin(c, T_STREAM, st2);
        if ((e = qs_launch_stream(&sa, grid, sn_smem, st2)) != cudaSuccess)
            return cuda_fail(c, e, "stream kernel launch");
        t_end(c, T_STREAM, st2);
    }
    if (n_live > 0) {
        // the rows the live-list kernel returned after the first cluster
        // launch stopped taking rows (clusters find nothing left and leave)
        if ((e = cudaEventRecord(c->join2, c->aux2)) != cudaSuccess || (e = cudaStreamWaitEvent(st, c->join2, 0)) != cudaSuccess)
            return cuda_fail(c, e, "join from the third stream");
        qs::QsLaunch ca = a;
        ca.rows = c->rows.p;
        ca.nrows = 0;
        ca.nrows_dev = nullptr;
        ca.n_s = plan.n_s;
        ca.lv_serve_returns = 1;
        e = qs_launch_rows(&ca, plan.clusters, plan.cl, plan.smem, st);
        if (e != cudaSuccess) return cuda_fail(c, e, "selection kernel launch (returned rows)");
        c->ctr.kernel_launches += 1;
    }
    if (both) {
        if ((e = cudaEventRecord(c->join, st2)) != cudaSuccess || (e = cudaStreamWaitEvent(st, c->join, 0)) != cudaSuccess)
            return cuda_fail(c, e, "join from the second stream");
    }
    c->ctr.calls += 1;
    c->ctr.rows += (uint64_t)B;
    c->ctr.logit_bytes += (uint64_t)B * (uint64_t)b->V * esz;
    c->ctr.last_stream_rows = n_stream;
    c->ctr.last_cluster_rows = n_cluster;
    c->ctr.last_hist_rows = n_hist;
    c->ctr.last_live_candidates = n_live;
    return mirror_status(c, st);
}

qsamp_status qsamp_sample(qsamp_ctx* c, const qsamp_batch* b, void* stream) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    qsamp_status s = sample_locked(c, b, (cudaStream_t)stream);
    if (prev != c->device) cudaSetDevice(prev);
    return s;
}

qsamp_status qsamp_sample_host(qsamp_ctx* c, const qsamp_batch* hb) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    qsamp_status s = validate(c, hb);
    if (s != QSAMP_OK || hb->B == 0) return s;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    const auto t0 = std::chrono::steady_clock::now();
    cudaStream_t st = c->stream;
    const int B = hb->B, V = hb->V;
    const size_t esz = hb->dtype == QSAMP_BF16 ? 2 : 4;
    qsamp_batch db = *hb;
    cudaError_t e;
    // Large batches: the logits cross PCIe in row chunks on the copy stream
    // while the kernels already run; a kernel takes a row once its chunk's
    // ready flag is set (the flag copy follows the chunk's copy in stream
    // order). Small batches: one copy before the kernels. Six chunks: each
    // flag copy stalls the copy engine (measured about 60 us per extra chunk
    // at B=256, V=151936), while fewer chunks leave a longer compute tail
    // after the last one lands (2 / 4 / 6 / 8 / 16 / 32 chunks: 82.1 / 82.9 /
    // 83.3 / 82.8 / 80.0 / 59.8 K rows/s end to end on one B200).
    const size_t total_bytes = (size_t)B * V * esz;
    const int nchunks = (B >= 32 && total_bytes >= ((size_t)16 << 20)) ? 6 : 1;
    const int chunk_rows = (B + nchunks - 1) / nchunks;
    const int* ready = nullptr;
    do {
        if ((e = c->h_logits.ensure((size_t)B * V * esz)) != cudaSuccess) break;
        if (nchunks == 1) {
            if ((e = cudaMemcpy2DAsync(c->h_logits.p, (size_t)V * esz, hb->logits, (size_t)hb->row_stride * esz,
                                       (size_t)V * esz, (size_t)B, cudaMemcpyHostToDevice, st)) != cudaSuccess)
                break;
        } else {
            if ((e = c->ready.ensure(nchunks)) != cudaSuccess) break;
            if ((e = cudaMemsetAsync(c->ready.p, 0, sizeof(int) * nchunks, st)) != cudaSuccess) break;
            // the copies start after the flags are cleared (and after the
            // previous call's work on st, which read the staging buffer)
            if ((e = cudaEventRecord(c->copy_go, st)) != cudaSuccess) break;
            if ((e = cudaStreamWaitEvent(c->copy, c->copy_go, 0)) != cudaSuccess) break;
            for (int j = 0; j < nchunks && e == cudaSuccess; ++j) {
                const int r0 = j * chunk_rows;
                const int nr = B - r0 < chunk_rows ? B - r0 : chunk_rows;
                if (nr <= 0) break;
                e = cudaMemcpy2DAsync((unsigned char*)c->h_logits.p + (size_t)r0 * V * esz, (size_t)V * esz,
                                      (const unsigned char*)hb->logits + (size_t)r0 * hb->row_stride * esz,
                                      (size_t)hb->row_stride * esz, (size_t)V * esz, (size_t)nr,
                                      cudaMemcpyHostToDevice, c->copy);
                // (fault injection for tests: chunks from drop_ready_from on
                // never raise their flag)
                if (e == cudaSuccess && (c->drop_ready_from < 0 || j < c->drop_ready_from))
                    e = cudaMemcpyAsync(c->ready.p + j, c->pinned_one, sizeof(int), cudaMemcpyHostToDevice, c->copy);
            }
            if (e != cudaSuccess) break;
            if ((e = cudaEventRecord(c->copy_done, c->copy)) != cudaSuccess) break;
            ready = c->ready.p;
        }
        db.logits = c->h_logits.p;
        db.row_stride = V;
        if (hb->hist) {
            if ((e = c->h_hist.ensure((size_t)B * hb->hist_stride)) != cudaSuccess) break;
            if ((e = cudaMemcpyAsync(c->h_hist.p, hb->hist, sizeof(int32_t) * (size_t)B * hb->hist_stride,
                                     cudaMemcpyHostToDevice, st)) != cudaSuccess)
                break;
            db.hist = c->h_hist.p;
        }
        if (hb->masks) {
            const size_t words = (size_t)(V + 31) / 32;
            const size_t rows = hb->mask_stride == 0 ? 1 : (size_t)B;
            const size_t stride = hb->mask_stride == 0 ? words : (size_t)hb->mask_stride;
            if ((e = c->h_masks.ensure(rows * stride)) != cudaSuccess) break;
            if ((e = cudaMemcpyAsync(c->h_masks.p, hb->masks, sizeof(uint32_t) * rows * stride, cudaMemcpyHostToDevice,
                                     st)) != cudaSuccess)
                break;
            db.masks = c->h_masks.p;
        }
        if ((e = c->h_ids.ensure(B)) != cudaSuccess) break;
        if ((e = c->h_results.ensure(B)) != cudaSuccess) break;
        db.out_ids = c->h_ids.p;
        db.out_results = c->h_results.p;
        if (hb->top_cap > 0) {
            if ((e = c->h_top_ids.ensure((size_t)B * hb->top_cap)) != cudaSuccess) break;
            if ((e = c->h_top_probs.ensure((size_t)B * hb->top_cap)) != cudaSuccess) break;
            db.out_top_ids = c->h_top_ids.p;
            db.out_top_probs = c->h_top_probs.p;
        }
    } while (0);
    if (e != cudaSuccess) {
        if (prev != c->device) cudaSetDevice(prev);
        return cuda_fail(c, e, "staging host inputs");
    }
    s = sample_locked(c, &db, st, ready, ready ? chunk_rows : 0);
    // st waits for the copy stream (flags and chunks) in every case
    if (ready) cudaStreamWaitEvent(st, c->copy_done, 0);
    if (s == QSAMP_OK) {
        do {
            if (hb->out_ids && (e = cudaMemcpyAsync(hb->out_ids, c->h_ids.p, sizeof(int32_t) * B,
                                                    cudaMemcpyDeviceToHost, st)) != cudaSuccess)
                break;
            if (hb->out_results && (e = cudaMemcpyAsync(hb->out_results, c->h_results.p,
                                                        sizeof(qsamp_row_result) * B, cudaMemcpyDeviceToHost, st)) !=
                                       cudaSuccess)
                break;
            if (hb->top_cap > 0) {
                if ((e = cudaMemcpyAsync(hb->out_top_ids, c->h_top_ids.p, sizeof(int32_t) * (size_t)B * hb->top_cap,
                                         cudaMemcpyDeviceToHost, st)) != cudaSuccess)
                    break;
                if ((e = cudaMemcpyAsync(hb->out_top_probs, c->h_top_probs.p, sizeof(float) * (size_t)B * hb->top_cap,
                                         cudaMemcpyDeviceToHost, st)) != cudaSuccess)
                    break;
            }
            e = cudaStreamSynchronize(st);
        } while (0);
        if (e != cudaSuccess) s = cuda_fail(c, e, "selection / copy back");
        else s = read_status(c);
    }
    c->ctr.last_call_us =
        std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
    if (prev != c->device) cudaSetDevice(prev);
    return s;
}

qsamp_status qsamp_poll_status(qsamp_ctx* c) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    return status_of(c, *(volatile int*)c->pinned_status);
}

qsamp_status qsamp_set_limits(qsamp_ctx* c, const qsamp_limits* l) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    if (!l) return fail(c, QSAMP_ERR_INVALID_ARG, "limits: expected non-NULL");
    if (l->max_rounds < 1)
        return fail(c, QSAMP_ERR_INVALID_ARG, "limits.max_rounds: expected >= 1, got %d", l->max_rounds);
    if (l->ready_wait_ns < 1000)
        return fail(c, QSAMP_ERR_INVALID_ARG, "limits.ready_wait_ns: expected >= 1000, got %lld",
                    (long long)l->ready_wait_ns);
    if (l->drop_ready_from < -1)
        return fail(c, QSAMP_ERR_INVALID_ARG, "limits.drop_ready_from: expected >= -1, got %d", l->drop_ready_from);
    if (l->hist_path != 0 && l->hist_path != 1)
        return fail(c, QSAMP_ERR_INVALID_ARG, "limits.hist_path: expected 0 or 1, got %d", l->hist_path);
    if (l->live_path < 0 || l->live_path > 2)
        return fail(c, QSAMP_ERR_INVALID_ARG, "limits.live_path: expected 0, 1 or 2, got %d", l->live_path);
    c->max_rounds = l->max_rounds;
    c->ready_wait_ns = (unsigned long long)l->ready_wait_ns;
    c->drop_ready_from = l->drop_ready_from;
    c->use_hist = l->hist_path != 0;
    c->use_live = l->live_path;
    return QSAMP_OK;
}

qsamp_status qsamp_get_limits(const qsamp_ctx* c, qsamp_limits* out) {
    if (!c || !out) return QSAMP_ERR_INVALID_ARG;
    out->max_rounds = c->max_rounds;
    out->ready_wait_ns = (int64_t)c->ready_wait_ns;
    out->drop_ready_from = c->drop_ready_from;
    out->hist_path = c->use_hist ? 1 : 0;
    out->live_path = c->use_live;
    return QSAMP_OK;
}

qsamp_status qsamp_get_counters(const qsamp_ctx* c, qsamp_counters* out) {
    if (!c || !out) return QSAMP_ERR_INVALID_ARG;
    *out = c->ctr;
    out->last_hist_handed_on = c->ctr.last_hist_rows > 0 ? ((volatile int*)c->pinned_status)[4] : 0;
    out->last_live_returned = c->live_last ? ((volatile int*)c->pinned_status)[5] : 0;
    out->last_live_rows = c->live_last ? ((volatile int*)c->pinned_status)[6] : 0;
    if (c->timing) {
        int prev = 0;
        cudaGetDevice(&prev);
        if (prev != c->device) cudaSetDevice(c->device);
        double* dst[5] = {&out->last_stream_kernel_ms, &out->last_rows_kernel_ms, &out->last_merge_kernel_ms,
                          &out->last_hist_kernel_ms, &out->last_live_kernel_ms};
        for (int k = 0; k < 5; ++k) {
            *dst[k] = 0.0;
            float ms = 0.0f;
            if (c->ev_used[k] && cudaEventSynchronize(c->ev[2 * k + 1]) == cudaSuccess &&
                cudaEventElapsedTime(&ms, c->ev[2 * k], c->ev[2 * k + 1]) == cudaSuccess)
                *dst[k] = ms;
        }
        if (prev != c->device) cudaSetDevice(prev);
    }
    return QSAMP_OK;
}

qsamp_status qsamp_set_kernel_timing(qsamp_ctx* c, int32_t on) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    qsamp_status s = QSAMP_OK;
    if (on && !c->ev[0]) {
        for (cudaEvent_t& ev : c->ev) {
            cudaError_t e = cudaEventCreate(&ev);
            if (e != cudaSuccess) {
                s = cuda_fail(c, e, "cudaEventCreate");
                break;
            }
        }
    }
    if (s == QSAMP_OK) c->timing = on != 0;
    for (bool& u : c->ev_used) u = false;
    if (prev != c->device) cudaSetDevice(prev);
    return s;
}

// ---------------------------------------------------------------- masks
qsamp_status qsamp_pack_ids(const int32_t* ids, int64_t n, int32_t V, uint32_t* mask_out) {
    if (V < 1 || !mask_out || (n > 0 && !ids) || n < 0) return QSAMP_ERR_INVALID_ARG;
    const int64_t words = (V + 31) / 32;
    std::memset(mask_out, 0, sizeof(uint32_t) * (size_t)words);
    for (int64_t i = 0; i < n; ++i) {
        const int32_t id = ids[i];
        if (id >= 0 && id < V) mask_out[id >> 5] |= 1u << (id & 31);
    }
    return QSAMP_OK;
}

qsamp_status qsamp_grammar_mask(const int32_t* valid_ids, int64_t n_valid, int32_t accepting, int32_t eos_string_id,
                                int32_t eos_token_id, int32_t V, uint32_t* mask_out, int32_t* force_token_out) {
    if (V < 1 || !mask_out || !force_token_out || n_valid < 0 || (n_valid > 0 && !valid_ids))
        return QSAMP_ERR_INVALID_ARG;
    const int64_t words = (V + 31) / 32;
    std::memset(mask_out, 0, sizeof(uint32_t) * (size_t)words);
    *force_token_out = -1;
    if (n_valid == 0) {
        // stuck grammar: every logit -inf except the first EOS string's (0.0)
        *force_token_out = (eos_string_id >= 0 && eos_string_id < V) ? eos_string_id : -1;
        return QSAMP_OK;
    }
    for (int64_t i = 0; i < n_valid; ++i) {
        const int32_t id = valid_ids[i];
        if (id >= 0 && id < V) mask_out[id >> 5] |= 1u << (id & 31);
    }
    if (accepting) {
        if (eos_string_id >= 0 && eos_string_id < V) mask_out[eos_string_id >> 5] |= 1u << (eos_string_id & 31);
        if (eos_token_id >= 0 && eos_token_id < V) mask_out[eos_token_id >> 5] |= 1u << (eos_token_id & 31);
    }
    return QSAMP_OK;
}

int32_t qsamp_find_eos_string(const char* const* strs, const int32_t* lens, int32_t V) {
    if (!strs || !lens) return -1;
    static const char a[] = "<|endoftext|>", b[] = "<|im_end|>";
    for (int32_t i = 0; i < V; ++i) {
        const int32_t n = lens[i];
        if (!strs[i]) continue;
        if ((n == (int32_t)sizeof(a) - 1 && std::memcmp(strs[i], a, (size_t)n) == 0) ||
            (n == (int32_t)sizeof(b) - 1 && std::memcmp(strs[i], b, (size_t)n) == 0))
            return i;
    }
    return -1;
}

qsamp_status qsamp_keep_list_mask(const char* path, int32_t V, uint32_t* mask_out) {
    if (!path || V < 1 || !mask_out) return QSAMP_ERR_INVALID_ARG;
    FILE* f = std::fopen(path, "rb");
    if (!f) return QSAMP_ERR_IO;
    uint32_t count = 0;
    if (std::fread(&count, sizeof count, 1, f) != 1) {
        std::fclose(f);
        return QSAMP_ERR_IO;
    }
    const int64_t words = (V + 31) / 32;
    std::memset(mask_out, 0, sizeof(uint32_t) * (size_t)words);
    for (uint32_t i = 0; i < count; ++i) {
        uint32_t id = 0;
        if (std::fread(&id, sizeof id, 1, f) != 1) {
            std::fclose(f);
            return QSAMP_ERR_IO;
        }
        const int32_t sid = (int32_t)id;
        if (sid >= 0 && sid < V) mask_out[sid >> 5] |= 1u << (sid & 31);
    }
    std::fclose(f);
    return QSAMP_OK;
}

qsamp_status qsamp_mask_and(const uint32_t* a, const uint32_t* b, int64_t words, uint32_t* out) {
    if (!a || !b || !out || words < 0) return QSAMP_ERR_INVALID_ARG;
    for (int64_t i = 0; i < words; ++i) out[i] = a[i] & b[i];
    return QSAMP_OK;
}

qsamp_status qsamp_verify_greedy(qsamp_ctx* c, const void* logits, qsamp_dtype dtype, int32_t V, int64_t row_stride,
                                 int32_t n_rows, int32_t B, const int32_t* row_off, const int32_t* drafts,
                                 int32_t eos_token, int32_t* out_accepted, int32_t* out_bonus,
                                 int32_t* out_has_bonus, void* stream) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    if (V < 1) return fail(c, QSAMP_ERR_INVALID_ARG, "V: expected >= 1, got %d", V);
    if (row_stride < V)
        return fail(c, QSAMP_ERR_INVALID_ARG, "row_stride: expected >= V (%d), got %lld", V, (long long)row_stride);
    if (dtype != QSAMP_F32 && dtype != QSAMP_BF16)
        return fail(c, QSAMP_ERR_INVALID_ARG, "dtype: expected QSAMP_F32 or QSAMP_BF16, got %d", (int)dtype);
    if (n_rows < 0 || B < 0) return fail(c, QSAMP_ERR_INVALID_ARG, "n_rows / B: expected >= 0, got %d / %d", n_rows, B);
    if (B == 0) return QSAMP_OK;
    if (!row_off || !out_accepted || !out_bonus || !out_has_bonus || (n_rows > 0 && (!logits || !drafts)))
        return fail(c, QSAMP_ERR_INVALID_ARG, "row_off / drafts / logits / outputs: expected non-NULL");
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    int segs = n_rows > 0 ? (2 * c->num_sms + n_rows - 1) / n_rows : 1;
    segs = segs < 1 ? 1 : (segs > 64 ? 64 : segs);
    cudaError_t e = c->vparts.ensure((size_t)(n_rows > 0 ? n_rows : 1) * segs);
    if (e == cudaSuccess)
        e = qs_launch_verify(logits, (int)dtype, V, row_stride, n_rows, B, row_off, drafts, eos_token, out_accepted,
                             out_bonus, out_has_bonus, c->vparts.p, segs, (cudaStream_t)stream);
    if (e == cudaSuccess) c->ctr.kernel_launches += n_rows > 0 ? 2 : 1;
    if (prev != c->device) cudaSetDevice(prev);
    return e == cudaSuccess ? QSAMP_OK : cuda_fail(c, e, "greedy verification launch");
}

qsamp_status qsamp_first_byte_table(const char* const* strs, const int32_t* lens, int32_t V, uint16_t* table_out) {
    if (V < 1 || !strs || !lens || !table_out) return QSAMP_ERR_INVALID_ARG;
    for (int32_t i = 0; i < V; ++i)
        table_out[i] = (lens[i] > 0 && strs[i]) ? (uint16_t)(unsigned char)strs[i][0] : (uint16_t)256;
    return QSAMP_OK;
}

qsamp_status qsamp_char_class_masks(qsamp_ctx* c, const uint16_t* table, int32_t V, int32_t B,
                                    const uint32_t* classes, uint32_t* masks, int64_t mask_stride, int32_t or_into,
                                    void* stream) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    if (V < 1) return fail(c, QSAMP_ERR_INVALID_ARG, "V: expected >= 1, got %d", V);
    if (B < 0 || B > 65535) return fail(c, QSAMP_ERR_INVALID_ARG, "B: expected [0,65535], got %d", B);
    if (B == 0) return QSAMP_OK;
    if (!table || !classes || !masks) return fail(c, QSAMP_ERR_INVALID_ARG, "table/classes/masks: expected non-NULL");
    const long long words = (V + 31) / 32;
    if (mask_stride < words)
        return fail(c, QSAMP_ERR_INVALID_ARG, "mask_stride: expected >= %lld words, got %lld", words,
                    (long long)mask_stride);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    cudaError_t e = qs_launch_char_class(table, V, B, classes, masks, mask_stride, or_into ? 1 : 0, c->num_sms,
                                         (cudaStream_t)stream);
    if (e == cudaSuccess) c->ctr.kernel_launches += 1;
    if (prev != c->device) cudaSetDevice(prev);
    return e == cudaSuccess ? QSAMP_OK : cuda_fail(c, e, "char-class mask launch");
}

// ---------------------------------------------------------------- sharded
// Candidates per row exchanged between ranks (n_ranks * k) are held by one
// CTA of the merge kernel.
static constexpr int kMergeCap = 5120;

static qsamp_status shard_locked(qsamp_ctx* c, const qsamp_batch* lb, int32_t v_offset, int32_t V_total, int32_t k,
                                 float* cand_vals, int32_t* cand_ids, cudaStream_t st) {
    if (!lb) return fail(c, QSAMP_ERR_INVALID_ARG, "local_batch: expected non-NULL");
    if (lb->V < 1) return fail(c, QSAMP_ERR_INVALID_ARG, "V (local): expected >= 1, got %d", lb->V);
    if (v_offset < 0) return fail(c, QSAMP_ERR_INVALID_ARG, "v_offset: expected >= 0, got %d", v_offset);
    if ((long long)V_total < (long long)v_offset + lb->V)
        return fail(c, QSAMP_ERR_INVALID_ARG, "V_total: expected >= v_offset + V (%lld), got %d",
                    (long long)v_offset + lb->V, V_total);
    if (k < 1 || k > qs::KMAX) return fail(c, QSAMP_ERR_INVALID_ARG, "k: expected [1,%d], got %d", qs::KMAX, k);
    if (!cand_vals || !cand_ids) return fail(c, QSAMP_ERR_INVALID_ARG, "cand_vals/cand_ids: expected non-NULL");
    qsamp_status s = validate(c, lb, V_total);
    if (s != QSAMP_OK || lb->B == 0) return s;
    const int B = lb->B;
    for (int r = 0; r < B; ++r) {
        const qsamp_row_params& p = lb->params[r];
        if (p.temperature > 0.0f && !(p.top_k > 0 && p.top_k <= k && p.top_k < V_total))
            return fail(c, QSAMP_ERR_UNSUPPORTED,
                        "params[%d].top_k: the sharded path serves 0 < top_k <= k (%d) and < V_total (%d), got %d "
                        "(a full-vocabulary top-p needs the unsharded path)", r, k, V_total, p.top_k);
        if (lb->hist) {
            const int len = lb->hist_len ? lb->hist_len[r] : lb->hist_stride;
            const bool pen = p.repetition_penalty != 1.0f || p.frequency_penalty != 0.0f || p.presence_penalty != 0.0f;
            const unsigned long long lbk = (unsigned long long)(long long)p.repetition_lookback;
            const long long w = (long long)(lbk < (unsigned long long)len ? lbk : (unsigned long long)len);
            if (pen && w > 1024)
                return fail(c, QSAMP_ERR_UNSUPPORTED, "row %d: the sharded path serves penalty windows <= 1024, got %lld",
                            r, w);
        }
    }
    const size_t sn_smem = qs_stream_smem(lb->V);
    if (c->max_dyn == 0) {
        size_t stc = 0;
        cudaError_t e0 = qs_kernel_static_smem(&stc);
        if (e0 != cudaSuccess) return cuda_fail(c, e0, "cudaFuncGetAttributes");
        c->max_dyn = (size_t)c->smem_optin - stc;
    }
    if (sn_smem > c->max_dyn)
        return fail(c, QSAMP_ERR_UNSUPPORTED, "V (local) = %d: the shard's allow-bitmap does not fit shared memory",
                    lb->V);
    qs::QsLaunch a;
    s = common_setup(c, lb, st, a);
    if (s != QSAMP_OK) return s;
    cudaError_t e;
    c->h_rows.resize((size_t)B);
    for (int r = 0; r < B; ++r) c->h_rows[(size_t)r] = r;
    if ((e = c->rows.ensure(B)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(rows)");
    if ((e = cudaMemcpyAsync(c->rows.p, c->h_rows.data(), sizeof(int32_t) * B, cudaMemcpyHostToDevice, st)) !=
        cudaSuccess)
        return cuda_fail(c, e, "copying row lists");
    if (sn_smem > c->stream_attr) {
        if ((e = qs_stream_attrs(sn_smem)) != cudaSuccess) return cuda_fail(c, e, "stream kernel attributes");
        c->stream_attr = sn_smem;
    }
    int per_sm = 0;
    if ((e = qs_stream_occupancy(sn_smem, &per_sm)) != cudaSuccess || per_sm <= 0)
        return cuda_fail(c, e == cudaSuccess ? cudaErrorInvalidConfiguration : e, "stream kernel occupancy");
    a.rows = c->rows.p;
    a.nrows = B;
    a.v_offset = v_offset;
    a.V_total = V_total;
    a.cand_vals = cand_vals;
    a.cand_ids = cand_ids;
    a.cand_k = k;
    const int grid = B < per_sm * c->num_sms ? B : per_sm * c->num_sms;
    for (bool& u : c->ev_used) u = false;
    t_begin(c, T_STREAM, st);
    if ((e = qs_launch_stream(&a, grid, sn_smem, st)) != cudaSuccess) return cuda_fail(c, e, "stream kernel launch");
    t_end(c, T_STREAM, st);
    c->ctr.calls += 1;
    c->ctr.rows += (uint64_t)B;
    c->ctr.logit_bytes += (uint64_t)B * (uint64_t)lb->V * (lb->dtype == QSAMP_BF16 ? 2 : 4);
    return mirror_status(c, st);
}

qsamp_status qsamp_shard_topk(qsamp_ctx* c, const qsamp_batch* lb, int32_t v_offset, int32_t V_total, int32_t k,
                              float* cand_vals, int32_t* cand_ids, void* stream) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    qsamp_status s = shard_locked(c, lb, v_offset, V_total, k, cand_vals, cand_ids, (cudaStream_t)stream);
    if (prev != c->device) cudaSetDevice(prev);
    return s;
}

static qsamp_status merge_locked(qsamp_ctx* c, int32_t n_ranks, int32_t B, int32_t k, const float* all_vals,
                                 const int32_t* all_ids, const qsamp_row_params* params, const double* u,
                                 uint64_t rng_offset, int32_t* out_ids, qsamp_row_result* out_results,
                                 cudaStream_t st) {
    if (n_ranks < 1) return fail(c, QSAMP_ERR_INVALID_ARG, "n_ranks: expected >= 1, got %d", n_ranks);
    if (B < 0) return fail(c, QSAMP_ERR_INVALID_ARG, "B: expected >= 0, got %d", B);
    if (k < 1 || k > qs::KMAX) return fail(c, QSAMP_ERR_INVALID_ARG, "k: expected [1,%d], got %d", qs::KMAX, k);
    if ((long long)n_ranks * k > kMergeCap)
        return fail(c, QSAMP_ERR_UNSUPPORTED, "n_ranks * k: expected <= %d candidates per row, got %lld", kMergeCap,
                    (long long)n_ranks * k);
    if (B == 0) return QSAMP_OK;
    if (!all_vals || !all_ids) return fail(c, QSAMP_ERR_INVALID_ARG, "all_vals/all_ids: expected non-NULL");
    if (!params) return fail(c, QSAMP_ERR_INVALID_ARG, "params: expected non-NULL");
    if (!out_ids && !out_results)
        return fail(c, QSAMP_ERR_INVALID_ARG, "out_ids/out_results: expected at least one non-NULL");
    for (int r = 0; r < B; ++r) {
        const qsamp_row_params& p = params[r];
        if (p.flags != 0) return fail(c, QSAMP_ERR_INVALID_ARG, "params[%d].flags: expected 0, got %d", r, p.flags);
        if (std::isnan(p.temperature))
            return fail(c, QSAMP_ERR_INVALID_ARG, "params[%d].temperature: expected a number, got NaN", r);
        if (p.temperature > 0.0f && !(p.top_k > 0 && p.top_k <= k))
            return fail(c, QSAMP_ERR_INVALID_ARG, "params[%d].top_k: expected (0,%d] for a merged row, got %d", r, k,
                        p.top_k);
        if (u && !(u[r] >= 0.0 && u[r] < 1.0))
            return fail(c, QSAMP_ERR_INVALID_ARG, "u[%d]: expected [0,1), got %g", r, u[r]);
    }
    cudaError_t e;
    if ((e = c->params.ensure(B)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(params)");
    if ((e = c->results.ensure(B)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(results)");
    if ((e = cudaMemcpyAsync(c->params.p, params, sizeof(qsamp_row_params) * B, cudaMemcpyHostToDevice, st)) !=
        cudaSuccess)
        return cuda_fail(c, e, "copying params");
    const double* d_u = nullptr;
    if (u) {
        if ((e = c->u.ensure(B)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(u)");
        if ((e = cudaMemcpyAsync(c->u.p, u, sizeof(double) * B, cudaMemcpyHostToDevice, st)) != cudaSuccess)
            return cuda_fail(c, e, "copying u");
        d_u = c->u.p;
    }
    if ((e = cudaMemsetAsync(c->status.p, 0, 2 * sizeof(int), st)) != cudaSuccess) return cuda_fail(c, e, "status reset");
    qs::QsLaunch a = {};
    a.B = B;
    a.params = c->params.p;
    a.u = d_u;
    a.philox_offset = rng_offset;
    a.results = out_results ? out_results : c->results.p;
    a.out_ids = out_ids;
    a.status = c->status.p;
    const size_t smem = qs_merge_smem();
    if (!c->merge_attr) {
        if ((e = qs_merge_attrs(smem)) != cudaSuccess) return cuda_fail(c, e, "merge kernel attributes");
        c->merge_attr = true;
    }
    const int grid = B < 2 * c->num_sms ? B : 2 * c->num_sms;
    for (bool& u : c->ev_used) u = false;
    t_begin(c, T_MERGE, st);
    if ((e = qs_launch_merge(&a, all_vals, all_ids, n_ranks, k, grid, smem, st)) != cudaSuccess)
        return cuda_fail(c, e, "merge kernel launch");
    t_end(c, T_MERGE, st);
    return mirror_status(c, st);
}

qsamp_status qsamp_merge_topk(qsamp_ctx* c, int32_t n_ranks, int32_t B, int32_t k, const float* all_vals,
                              const int32_t* all_ids, const qsamp_row_params* params, const double* u,
                              uint64_t rng_offset, int32_t* out_ids, qsamp_row_result* out_results, void* stream) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    qsamp_status s = merge_locked(c, n_ranks, B, k, all_vals, all_ids, params, u, rng_offset, out_ids, out_results,
                                  (cudaStream_t)stream);
    if (prev != c->device) cudaSetDevice(prev);
    return s;
}

}  // extern "C"
