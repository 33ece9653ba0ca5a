// qsamp_static.cu -- qsamp_sample_static: the batched selection without any
// device allocation.
//
// Who needs it: callers that cannot allocate device memory at the point
// where they sample -- a serving engine whose device memory is fully
// reserved up front by its own allocator, or a plugin host that forbids its
// plugins to call cudaMalloc. qsamp_create() allocates (its scratch buffers
// and a stream), so those callers cannot hold a qsamp_ctx; this entry point
// needs none.
//
// Where the scratch lives instead: qs_static_scratch below, a file-scope
// __device__ array of QSAMP_STATIC_SCRATCH_BYTES (640 KiB). Every GPU
// that loads libqsamp.so holds one copy until the process exits. It stages
// the per-row parameters, history lengths, uniforms and results (up to
// QSAMP_STATIC_MAX_ROWS rows), the device status word and the cluster
// kernel's row queue, and one bf16 soft-cap table. A host pointer to it is
// obtained per device with cudaGetSymbolAddress -- the array's name in host
// code is only a stand-in, never a device address.
//
// Sharing rules: all calls on a device share the one array and it keeps the
// previous call's contents. Each call rewrites everything it reads (the
// status word and row queue are cleared, parameters and the soft-cap table are copied or
// rebuilt). Two calls whose work overlaps on the GPU (different streams, or
// different host threads) race on the array and must be serialised by the
// caller.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "qsamp_device.h"

extern "C" cudaError_t qs_launch_rows(const qs::QsLaunch* a, int clusters, int cl, size_t smem, cudaStream_t st);
extern "C" cudaError_t qs_kernel_attrs(size_t smem);
extern "C" cudaError_t qs_kernel_static_smem(size_t* out);
extern "C" cudaError_t qs_max_clusters(int cl, size_t smem, int* out);
extern "C" cudaError_t qs_launch_lut(float* lut, float cap, cudaStream_t st);

namespace {

constexpr size_t kStatusBytes = 256;
constexpr size_t kLutBytes = 65536 * sizeof(float);
constexpr size_t kParamsOff = kStatusBytes + kLutBytes;
constexpr size_t kHistLenOff = kParamsOff + (size_t)QSAMP_STATIC_MAX_ROWS * sizeof(qsamp_row_params);
constexpr size_t kUOff = kHistLenOff + (size_t)QSAMP_STATIC_MAX_ROWS * sizeof(int32_t);
constexpr size_t kResultsOff = kUOff + (size_t)QSAMP_STATIC_MAX_ROWS * sizeof(double);
constexpr size_t kTotal = kResultsOff + (size_t)QSAMP_STATIC_MAX_ROWS * sizeof(qsamp_row_result);
static_assert(kTotal <= QSAMP_STATIC_SCRATCH_BYTES, "static scratch layout exceeds its declared size");
static_assert(kParamsOff % 16 == 0 && kHistLenOff % 16 == 0 && kUOff % 16 == 0 && kResultsOff % 16 == 0,
              "static scratch regions must stay 16-byte aligned");

constexpr int kMaxDevices = 64;
constexpr int kMaxRounds = 64;

struct DevState {
    bool ready = false;
    unsigned char* scratch = nullptr;  // device address of qs_static_scratch on this device
    size_t max_dyn = 0;
};
DevState g_dev[kMaxDevices];
std::mutex g_mu;

qsamp_status report(char* err, size_t n, qsamp_status s, const char* fmt, ...) {
    if (err && n) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, n, fmt, ap);
        va_end(ap);
    }
    return s;
}

}  // namespace

// The scratch itself (see the file comment for its layout and sharing rules).
static __device__ __align__(256) unsigned char qs_static_scratch[QSAMP_STATIC_SCRATCH_BYTES];

extern "C" qsamp_status qsamp_sample_static(const qsamp_batch* b, void* stream, char* err, size_t err_len) {
    if (err && err_len) err[0] = '\0';
    if (!b) return report(err, err_len, QSAMP_ERR_INVALID_ARG, "batch: expected non-NULL");
    if (b->B < 0) return report(err, err_len, QSAMP_ERR_INVALID_ARG, "B: expected >= 0, got %d", b->B);
    if (b->B == 0) return QSAMP_OK;
    if (b->B > QSAMP_STATIC_MAX_ROWS)
        return report(err, err_len, QSAMP_ERR_INVALID_ARG,
                      "B: the allocation-free entry point serves at most %d rows per call, got %d",
                      QSAMP_STATIC_MAX_ROWS, b->B);
    if (b->V < 1) return report(err, err_len, QSAMP_ERR_INVALID_ARG, "V: expected >= 1, got %d", b->V);
    if (b->row_stride < b->V)
        return report(err, err_len, QSAMP_ERR_INVALID_ARG, "row_stride: expected >= V (%d), got %lld", b->V,
                      (long long)b->row_stride);
    if (!b->logits || !b->params)
        return report(err, err_len, QSAMP_ERR_INVALID_ARG, "logits/params: expected non-NULL");
    if (b->dtype != QSAMP_F32 && b->dtype != QSAMP_BF16)
        return report(err, err_len, QSAMP_ERR_INVALID_ARG, "dtype: expected QSAMP_F32 or QSAMP_BF16");
    if (!b->out_ids && !b->out_results)
        return report(err, err_len, QSAMP_ERR_INVALID_ARG, "out_ids/out_results: expected at least one non-NULL");
    if (b->top_cap < 0 || b->top_cap > qs::KMAX || (b->top_cap > 0 && (!b->out_top_ids || !b->out_top_probs)))
        return report(err, err_len, QSAMP_ERR_INVALID_ARG, "top_cap: expected [0,%d] with both top outputs",
                      qs::KMAX);
    if (b->hist && b->hist_stride < 1)
        return report(err, err_len, QSAMP_ERR_INVALID_ARG, "hist_stride: expected >= 1 with hist");
    const long long words = (b->V + 31) / 32;
    if (b->masks && b->mask_stride != 0 && b->mask_stride < words)
        return report(err, err_len, QSAMP_ERR_INVALID_ARG, "mask_stride: expected 0 or >= %lld words", words);
    for (int r = 0; r < b->B; ++r) {
        const qsamp_row_params& p = b->params[r];
        if (p.flags != 0 || p.temperature != p.temperature || p.force_token < -1 || p.force_token >= b->V)
            return report(err, err_len, QSAMP_ERR_INVALID_ARG, "params[%d]: flags, temperature or force_token invalid",
                          r);
        if (b->hist) {
            const int len = b->hist_len ? b->hist_len[r] : b->hist_stride;
            if (len < 0 || len > b->hist_stride)
                return report(err, err_len, QSAMP_ERR_INVALID_ARG, "hist_len[%d]: expected [0,%d], got %d", r,
                              b->hist_stride, len);
            const bool pen = p.repetition_penalty != 1.0f || p.frequency_penalty != 0.0f || p.presence_penalty != 0.0f;
            const unsigned long long lb = (unsigned long long)(long long)p.repetition_lookback;
            const long long w = (long long)(lb < (unsigned long long)len ? lb : (unsigned long long)len);
            if (pen && w > qs::HIST_MAX)
                return report(err, err_len, QSAMP_ERR_UNSUPPORTED, "row %d: penalty window of %lld ids exceeds %d", r,
                              w, qs::HIST_MAX);
        }
        if (b->u && !(b->u[r] >= 0.0 && b->u[r] < 1.0))
            return report(err, err_len, QSAMP_ERR_INVALID_ARG, "u[%d]: expected [0,1)", r);
    }

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return report(err, err_len, QSAMP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return report(err, err_len, QSAMP_ERR_UNSUPPORTED, "device %d", dev);
    std::lock_guard<std::mutex> g(g_mu);
    DevState& d = g_dev[dev];
    if (!d.ready) {
        // once per device, with that device current: the scratch array's
        // device address (the host-side name is not one), and the kernel's
        // shared-memory limit
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, qs_static_scratch);
        if (e != cudaSuccess)
            return report(err, err_len, QSAMP_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        int optin = 0;
        e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        size_t st = 0;
        if (e == cudaSuccess) e = qs_kernel_static_smem(&st);
        if (e == cudaSuccess) e = qs_kernel_attrs((size_t)optin - st);
        if (e != cudaSuccess) return report(err, err_len, QSAMP_ERR_CUDA, "set-up: %s", cudaGetErrorString(e));
        d.scratch = (unsigned char*)ptr;
        d.max_dyn = (size_t)optin - st;
        d.ready = true;
    }
    cudaStream_t s = (cudaStream_t)stream;
    unsigned char* base = d.scratch;
    int* status = (int*)base;
    float* lut = (float*)(base + kStatusBytes);
    qsamp_row_params* d_params = (qsamp_row_params*)(base + kParamsOff);
    int32_t* d_hl = (int32_t*)(base + kHistLenOff);
    double* d_u = (double*)(base + kUOff);
    qsamp_row_result* d_res = (qsamp_row_result*)(base + kResultsOff);
    const int B = b->B;

    // the previous call's contents: clear the status, rewrite what is read
    if ((e = cudaMemsetAsync(status, 0, 2 * sizeof(int), s)) != cudaSuccess ||
        (e = cudaMemcpyAsync(d_params, b->params, sizeof(qsamp_row_params) * B, cudaMemcpyHostToDevice, s)) !=
            cudaSuccess ||
        (b->hist && b->hist_len &&
         (e = cudaMemcpyAsync(d_hl, b->hist_len, sizeof(int32_t) * B, cudaMemcpyHostToDevice, s)) != cudaSuccess) ||
        (b->u && (e = cudaMemcpyAsync(d_u, b->u, sizeof(double) * B, cudaMemcpyHostToDevice, s)) != cudaSuccess))
        return report(err, err_len, QSAMP_ERR_CUDA, "staging into the static scratch: %s", cudaGetErrorString(e));
    float lut_cap = 0.0f;
    if (b->dtype == QSAMP_BF16) {
        for (int r = 0; r < B && lut_cap == 0.0f; ++r)
            if (b->params[r].softcap > 0.0f) lut_cap = b->params[r].softcap;
        if (lut_cap > 0.0f && (e = qs_launch_lut(lut, lut_cap, s)) != cudaSuccess)
            return report(err, err_len, QSAMP_ERR_CUDA, "soft-cap table: %s", cudaGetErrorString(e));
    }

    // launch plan: the smallest cluster whose slices fit, wider while every
    // row still has its own cluster
    const int sizes[5] = {1, 2, 4, 8, 16};
    int pick = -1;
    int clusters = 0;
    for (int i = 0; i < 5; ++i) {
        const int cl = sizes[i];
        const int n_s = qs::align_up((b->V + cl - 1) / cl, 8);
        const size_t smem = (size_t)qs::smem_layout(n_s).total;
        if (smem > d.max_dyn) continue;
        int mc = 0;
        if (qs_max_clusters(cl, smem, &mc) != cudaSuccess) {
            cudaGetLastError();
            mc = 0;
        }
        if (mc <= 0) {
            if (pick >= 0) break;
            continue;
        }
        if (pick < 0 || mc >= B) {
            pick = i;
            clusters = mc;
        }
        if (mc < B) break;
    }
    if (pick < 0)
        return report(err, err_len, QSAMP_ERR_UNSUPPORTED, "V=%d does not fit one 16-CTA cluster", b->V);
    const int cl = sizes[pick];
    qs::QsLaunch a = {};
    a.logits = b->logits;
    a.dtype = (int)b->dtype;
    a.B = B;
    a.V = b->V;
    a.row_stride = b->row_stride;
    const size_t esz = b->dtype == QSAMP_BF16 ? 2 : 4;
    a.vec_ok = ((uintptr_t)b->logits % 16 == 0) && ((size_t)b->row_stride * esz % 16 == 0);
    a.params = d_params;
    a.hist = b->hist;
    a.hist_stride = b->hist_stride;
    a.hist_len = (b->hist && b->hist_len) ? d_hl : nullptr;
    a.masks = b->masks;
    a.mask_stride = b->mask_stride;
    a.u = b->u ? d_u : nullptr;
    a.philox_offset = b->rng_offset;
    a.luts = lut_cap > 0.0f ? lut : nullptr;
    a.lut_caps[0] = lut_cap;
    a.results = b->out_results ? b->out_results : d_res;
    a.out_ids = b->out_ids;
    a.top_ids = b->top_cap > 0 ? b->out_top_ids : nullptr;
    a.top_probs = b->top_cap > 0 ? b->out_top_probs : nullptr;
    a.top_cap = b->top_cap;
    a.status = status;
    a.row_ctr = status + 1;  // the cluster kernel's row queue
    a.n_s = qs::align_up((b->V + cl - 1) / cl, 8);
    a.max_rounds = kMaxRounds;
    const size_t smem = (size_t)qs::smem_layout(a.n_s).total;
    e = qs_launch_rows(&a, clusters < B ? clusters : B, cl, smem, s);
    if (e != cudaSuccess) return report(err, err_len, QSAMP_ERR_CUDA, "selection kernel: %s", cudaGetErrorString(e));
    return QSAMP_OK;
}
