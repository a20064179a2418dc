// C ABI of the B200 quantized matvec library (declared in include/qmv_b200.h).
//
// Host-side duties: argument/view validation with the reference's rules
// (src/quantized_matvec.cpp:94-149, :168-191), upload + repack of packed
// tensors, the thread-safe residency registry keyed by the view's host data
// pointer, per-thread device staging for the host-pointer drop-in entry
// points, and error reporting (0 return + per-thread message; never abort).
#include <cuda_runtime.h>

#include <limits.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "qmv_b200.h"
#include "qmv_internal.h"

#define QMV_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_error;

int fail(const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_error = buf;
    return 0;
}

int cuda_fail(const char *what, cudaError_t e)
{
    return fail("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define QMV_CUDA(call, what)                         \
    do {                                             \
        cudaError_t e_ = (call);                     \
        if (e_ != cudaSuccess) return cuda_fail(what, e_); \
    } while (0)

// The reference's view checks for one matrix (quantized_matvec.cpp:94-149),
// without the input/output counts.  Fills rows/cols on success.
int check_view(const GgufQuantizedTensorView *m, int *rows_out, int *cols_out)
{
    if (m == nullptr || m->data == nullptr) return fail("matrix view or its data is null");
    if (m->dimension_count != 2) return fail("matrix view must have 2 dimensions");
    const uint64_t ncols = m->dimensions[0], nrows = m->dimensions[1];
    if (ncols == 0 || nrows == 0 || ncols > INT_MAX || nrows > INT_MAX)
        return fail("matrix dimensions must be in 1..INT_MAX");
    const int be = qmv::block_elements(m->ggml_type);
    const int bb = qmv::block_bytes(m->ggml_type);
    if (be == 0) return fail("unsupported GGML type %u (Q5_0, Q8_0, Q4_K and Q6_K only)", m->ggml_type);
    if (m->block_elements != (uint64_t)be || m->block_bytes != (uint64_t)bb || ncols % (uint64_t)be)
        return fail("block layout does not match GGML type %u", m->ggml_type);
    const uint64_t bpr = ncols / (uint64_t)be;
    if (bpr > UINT64_MAX / nrows || m->block_count != bpr * nrows || ncols > UINT64_MAX / nrows ||
        m->element_count != ncols * nrows || m->block_count > SIZE_MAX / (uint64_t)bb)
        return fail("block_count/element_count do not agree with the shape");
    *rows_out = (int)nrows;
    *cols_out = (int)ncols;
    return 1;
}

int current_device(int *dev)
{
    QMV_CUDA(cudaGetDevice(dev), "cudaGetDevice");
    return 1;
}

int check_weight(const QmvWeight *w)
{
    if (w == nullptr || w->dev == nullptr) return fail("weight handle is null");
    int dev = -1;
    if (!current_device(&dev)) return 0;
    if (dev != w->device)
        return fail("weight lives on device %d but the calling thread's device is %d", w->device, dev);
    return 1;
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

int upload(const GgufQuantizedTensorView *view, int row_begin, int row_end, QmvWeight **out)
{
    int rows = 0, cols = 0;
    if (out == nullptr) return fail("output handle pointer is null");
    *out = nullptr;
    if (!check_view(view, &rows, &cols)) return 0;
    if (cols > qmv::kMaxCols) return fail("%d columns exceed this build's limit of %d", cols, qmv::kMaxCols);
    if (row_begin < 0 || row_end > rows || row_begin >= row_end)
        return fail("row range [%d, %d) is outside 0..%d", row_begin, row_end, rows);
    int dev = 0;
    if (!current_device(&dev)) return 0;
    qmv::Layout L;
    if (!qmv::make_layout(view->ggml_type, row_end - row_begin, cols, &L)) return fail("bad layout");
    const uint64_t raw_row = (uint64_t)L.nb * (uint64_t)qmv::block_bytes(L.type);
    const uint64_t raw_bytes = raw_row * (uint64_t)L.rows;
    const size_t bytes = (size_t)L.row_stride * (size_t)L.rows;
    const unsigned char *src = view->data + raw_row * (uint64_t)row_begin;

    QmvWeight *w = new QmvWeight{L, nullptr, bytes, dev, row_begin, false};
    cudaStream_t s = nullptr;
    uint8_t *tmp = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&w->dev, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&tmp, raw_bytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, src, raw_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = qmv::launch_repack(L, tmp, w->dev, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (tmp) cudaFree(tmp);
    if (s) cudaStreamDestroy(s);
    if (e != cudaSuccess) {
        if (w->dev) cudaFree(w->dev);
        delete w;
        return cuda_fail("weight upload", e);
    }
    *out = w;
    return 1;
}

// ---------------------------------------------------------------- registry

typedef std::tuple<int, const void *, uint32_t, int, int> RegKey;
std::mutex g_reg_mutex;
std::map<RegKey, QmvWeight *> g_registry;

// ------------------------------------------------- per-thread staging

struct Staging {
    cudaStream_t stream = nullptr;
    float *dx = nullptr;
    size_t dx_cap = 0;
    float *dy = nullptr;
    size_t dy_cap = 0;
    void *ws = nullptr;
    unsigned long long *dkey = nullptr;
    unsigned long long *hkey = nullptr;
    unsigned int *hstatus = nullptr;  // mapped pinned word: this thread's expired-wait bits
    unsigned int *dstatus = nullptr;  // its device address
    cudaEvent_t ev[2] = {nullptr, nullptr};  // around the kernels (profiling)
};

struct StagingSet {
    std::map<int, Staging> per_device;
    ~StagingSet()
    {
        for (auto &kv : per_device) {
            Staging &st = kv.second;
            if (cudaSetDevice(kv.first) != cudaSuccess) continue;
            if (st.stream) {
                qmv::stream_free(st.dx, st.stream);
                qmv::stream_free(st.dy, st.stream);
                cudaStreamSynchronize(st.stream);
            }
            cudaFree(st.ws);
            cudaFree(st.dkey);
            cudaFreeHost(st.hkey);
            cudaFreeHost(st.hstatus);
            for (cudaEvent_t ev : st.ev)
                if (ev) cudaEventDestroy(ev);
            if (st.stream) cudaStreamDestroy(st.stream);
        }
    }
};

thread_local StagingSet g_staging;

// Per-thread kernel timing of the host-pointer drop-in calls: when on, each
// call brackets its kernels (not its copies) with events on its stream.
thread_local bool g_profiling = false;
thread_local double g_last_kernel_seconds = -1.0;

int kernels_begin(Staging *st)
{
    if (!g_profiling) return 1;
    for (cudaEvent_t &ev : st->ev)
        if (ev == nullptr) QMV_CUDA(cudaEventCreate(&ev), "cudaEventCreate");
    QMV_CUDA(cudaEventRecord(st->ev[0], st->stream), "cudaEventRecord");
    return 1;
}

int kernels_end(Staging *st)
{
    if (!g_profiling) return 1;
    QMV_CUDA(cudaEventRecord(st->ev[1], st->stream), "cudaEventRecord");
    return 1;
}

// After the call's synchronisation.
int kernels_elapsed(Staging *st)
{
    if (!g_profiling) return 1;
    float ms = 0.f;
    QMV_CUDA(cudaEventElapsedTime(&ms, st->ev[0], st->ev[1]), "cudaEventElapsedTime");
    g_last_kernel_seconds = (double)ms * 1e-3;
    return 1;
}

int staging(Staging **out)
{
    int dev = 0;
    if (!current_device(&dev)) return 0;
    Staging &st = g_staging.per_device[dev];
    if (st.stream == nullptr) {
        QMV_CUDA(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking), "cudaStreamCreate");
        QMV_CUDA(cudaMalloc(&st.ws, qmv::kArgmaxWorkspaceBytes), "cudaMalloc(workspace)");
        QMV_CUDA(cudaMemset(st.ws, 0, qmv::kArgmaxWorkspaceBytes), "cudaMemset(workspace)");
        QMV_CUDA(cudaMalloc(&st.dkey, sizeof(unsigned long long)), "cudaMalloc(key)");
        QMV_CUDA(cudaMallocHost(&st.hkey, sizeof(unsigned long long)), "cudaMallocHost(key)");
        QMV_CUDA(cudaHostAlloc(&st.hstatus, 16, cudaHostAllocMapped), "cudaHostAlloc(status)");
        QMV_CUDA(cudaHostGetDevicePointer((void **)&st.dstatus, st.hstatus, 0), "cudaHostGetDevicePointer");
    }
    *out = &st;
    return 1;
}

// Grow a per-thread staging buffer on its own stream from the library's
// stream-ordered pool: no cudaFree (and so no device-wide synchronisation)
// on the call path when a larger shape arrives.
int grow(float **buf, size_t *cap, size_t count, cudaStream_t s)
{
    if (*cap >= count) return 1;
    QMV_CUDA(qmv::stream_free(*buf, s), "free staging");
    *buf = nullptr;
    *cap = 0;
    QMV_CUDA(qmv::stream_alloc((void **)buf, count * sizeof(float), s), "allocate staging");
    *cap = count;
    return 1;
}

// For the duration of one drop-in call, the kernels this thread launches also
// report expired bounded waits in the thread's own status word.
struct CallStatus {
    Staging *st;
    explicit CallStatus(Staging *s) : st(s)
    {
        *st->hstatus = 0u;
        qmv::set_call_status(st->dstatus);
    }
    ~CallStatus() { qmv::set_call_status(nullptr); }
    // after the call's synchronisation
    int check(const char *what) const
    {
        const unsigned int v = *(volatile unsigned int *)st->hstatus;
        if (v != 0u) return fail("%s: a bounded wait of this call's kernel expired (status 0x%x)", what, v);
        return 1;
    }
};

int decode_key(unsigned long long key, int *id)
{
    if (key == QMV_KEY_NONFINITE || (key >> 32) == 0ull) {
        *id = -1;
        return 0;
    }
    *id = (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
    return 1;
}

}  // namespace

namespace qmv {
int set_error(const char *msg) { return fail("%s", msg); }

int release_resident_range(const void *begin, const void *end)
{
    std::lock_guard<std::mutex> lock(g_reg_mutex);
    int n = 0, prev = -1;
    for (auto it = g_registry.begin(); it != g_registry.end();) {
        const char *p = (const char *)std::get<1>(it->first);
        if (p < (const char *)begin || p >= (const char *)end) {
            ++it;
            continue;
        }
        if (prev < 0 && cudaGetDevice(&prev) != cudaSuccess) prev = 0;
        cudaSetDevice(it->second->device);
        cudaFree(it->second->dev);
        delete it->second;
        it = g_registry.erase(it);
        ++n;
    }
    if (prev >= 0) cudaSetDevice(prev);
    return n;
}
int set_cuda_error(const char *what, cudaError_t e) { return cuda_fail(what, e); }
}  // namespace qmv

// ================================================================ exported

QMV_EXPORT const char *qmv_last_error(void) { return g_error.c_str(); }

QMV_EXPORT int qmv_copy_last_error(char *buf, int capacity)
{
    if (buf == nullptr || capacity <= 0) return 0;
    snprintf(buf, (size_t)capacity, "%s", g_error.c_str());
    return 1;
}

QMV_EXPORT int qmv_abi_version(void) { return 1; }

QMV_EXPORT int qmv_device_count(int *count)
{
    if (count == nullptr) return fail("count pointer is null");
    *count = 0;
    QMV_CUDA(cudaGetDeviceCount(count), "cudaGetDeviceCount");
    return 1;
}

QMV_EXPORT int qmv_set_device(int device)
{
    QMV_CUDA(cudaSetDevice(device), "cudaSetDevice");
    return 1;
}

QMV_EXPORT int qmv_device_status(uint32_t *flags, int clear)
{
    if (flags == nullptr) return fail("flags pointer is null");
    unsigned int v = 0;
    QMV_CUDA(qmv::read_status(&v, clear != 0), "read device status");
    *flags = v;
    return 1;
}

QMV_EXPORT int qmv_set_gemv_path(int path)
{
    if (path < 0 || path > 5) return fail("gemv path must be 0, 1, 2, 3, 4 or 5");
    qmv::set_gemv_path(path);
    return 1;
}

QMV_EXPORT int qmv_set_profiling(int enabled)
{
    g_profiling = enabled != 0;
    g_last_kernel_seconds = -1.0;
    return 1;
}

QMV_EXPORT int qmv_last_kernel_seconds(double *seconds)
{
    if (seconds == nullptr) return fail("null output");
    if (g_last_kernel_seconds < 0.0) return fail("no profiled call on this thread (qmv_set_profiling(1) first)");
    *seconds = g_last_kernel_seconds;
    return 1;
}

QMV_EXPORT int qmv_set_matmul_path(int path)
{
    if (!(path == 0 || path == 1 || path == 2 || path == 64 || path == 128 || path == 176 || path == 256))
        return fail("matmul path must be 0, 1, 2, 64, 128, 176 or 256");
    qmv::set_matmul_path(path);
    return 1;
}

QMV_EXPORT int qmv_weight_upload(const GgufQuantizedTensorView *view, int row_begin, int row_end,
                                 QmvWeight **out)
{
    return upload(view, row_begin, row_end, out);
}

QMV_EXPORT int qmv_weight_free(QmvWeight *w)
{
    if (w == nullptr) return fail("weight handle is null");
    if (w->registry_owned) return fail("weight is owned by the residency registry");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(w->device);
    cudaError_t e = cudaFree(w->dev);
    cudaSetDevice(prev);
    delete w;
    if (e != cudaSuccess) return cuda_fail("cudaFree(weight)", e);
    return 1;
}

QMV_EXPORT int qmv_weight_info(const QmvWeight *w, uint32_t *type, int *rows, int *cols,
                               int *row_begin, uint64_t *device_bytes)
{
    if (w == nullptr) return fail("weight handle is null");
    if (type) *type = w->L.type;
    if (rows) *rows = w->L.rows;
    if (cols) *cols = w->L.cols;
    if (row_begin) *row_begin = w->row_begin;
    if (device_bytes) *device_bytes = w->bytes;
    return 1;
}

QMV_EXPORT int qmv_resident_weight(const GgufQuantizedTensorView *view, QmvWeight **out)
{
    int rows = 0, cols = 0, dev = 0;
    if (out == nullptr) return fail("output handle pointer is null");
    *out = nullptr;
    if (!check_view(view, &rows, &cols)) return 0;
    if (!current_device(&dev)) return 0;
    const RegKey key(dev, (const void *)view->data, view->ggml_type, rows, cols);
    std::lock_guard<std::mutex> lock(g_reg_mutex);
    auto it = g_registry.find(key);
    if (it != g_registry.end()) {
        *out = it->second;
        return 1;
    }
    QmvWeight *w = nullptr;
    if (!upload(view, 0, rows, &w)) return 0;
    w->registry_owned = true;
    g_registry[key] = w;
    *out = w;
    return 1;
}

QMV_EXPORT int qmv_resident_release_all(void)
{
    std::lock_guard<std::mutex> lock(g_reg_mutex);
    int prev = 0;
    cudaGetDevice(&prev);
    for (auto &kv : g_registry) {
        cudaSetDevice(kv.second->device);
        cudaFree(kv.second->dev);
        delete kv.second;
    }
    g_registry.clear();
    cudaSetDevice(prev);
    return 1;
}

QMV_EXPORT int qmv_matvec(const QmvWeight *w, const float *x, int x_count, float *y, int y_count,
                          void *stream)
{
    if (!check_weight(w)) return 0;
    if (x == nullptr || y == nullptr) return fail("x or y is null");
    if (x_count != w->L.cols || y_count != w->L.rows)
        return fail("counts (%d, %d) do not match the %d x %d weight", x_count, y_count, w->L.rows, w->L.cols);
    if (!aligned16(x)) return fail("x must be 16-byte aligned");
    QMV_CUDA(qmv::launch_gemv(w->L, w->dev, x, y, nullptr, (cudaStream_t)stream), "gemv launch");
    return 1;
}

QMV_EXPORT int qmv_matmul(const QmvWeight *w, const float *X, int x_count, int batch, float *Y,
                          int y_count, void *stream)
{
    if (!check_weight(w)) return 0;
    if (X == nullptr || Y == nullptr) return fail("X or Y is null");
    if (batch <= 0) return fail("batch must be positive");
    if (x_count != w->L.cols || y_count != w->L.rows)
        return fail("counts (%d, %d) do not match the %d x %d weight", x_count, y_count, w->L.rows, w->L.cols);
    if (!aligned16(X)) return fail("X must be 16-byte aligned");
    QMV_CUDA(qmv::launch_matmul(w->L, w->dev, X, batch, Y, (cudaStream_t)stream), "matmul launch");
    return 1;
}

QMV_EXPORT int qmv_matmul_residual(const QmvWeight *w, const float *X, int x_count, int batch, float *H,
                                   int h_count, void *stream)
{
    if (!check_weight(w)) return 0;
    if (X == nullptr || H == nullptr) return fail("X or H is null");
    if (batch <= 0) return fail("batch must be positive");
    if (x_count != w->L.cols || h_count != w->L.rows)
        return fail("counts (%d, %d) do not match the %d x %d weight", x_count, h_count, w->L.rows, w->L.cols);
    if (!aligned16(X)) return fail("X must be 16-byte aligned");
    QMV_CUDA(qmv::launch_matmul_residual(w->L, w->dev, X, batch, H, (cudaStream_t)stream), "matmul launch");
    return 1;
}

QMV_EXPORT int qmv_dequantize(const QmvWeight *w, float *out, uint64_t out_count, void *stream)
{
    if (!check_weight(w)) return 0;
    if (out == nullptr) return fail("out is null");
    if (out_count != (uint64_t)w->L.rows * (uint64_t)w->L.cols) return fail("out_count must be rows * cols");
    QMV_CUDA(qmv::launch_dequant_layout(w->L, w->dev, out, (cudaStream_t)stream), "dequant launch");
    return 1;
}

QMV_EXPORT int qmv_dequantize_raw(uint32_t type, const void *blocks, uint64_t block_count, float *out,
                                  void *stream)
{
    if (qmv::block_elements(type) == 0) return fail("unsupported GGML type %u", type);
    if (blocks == nullptr || out == nullptr) return fail("blocks or out is null");
    if (block_count == 0) return 1;
    QMV_CUDA(qmv::launch_dequant_raw(type, (const uint8_t *)blocks, block_count, out, (cudaStream_t)stream),
             "dequant launch");
    return 1;
}

QMV_EXPORT size_t qmv_argmax_workspace_bytes(void) { return qmv::kArgmaxWorkspaceBytes; }

QMV_EXPORT int qmv_argmax(const float *logits, int n, int index_base, uint64_t *key, void *workspace,
                          void *stream)
{
    if (logits == nullptr || key == nullptr || workspace == nullptr)
        return fail("logits, key or workspace is null");
    if (n <= 0) return fail("vocabulary size must be positive");
    if (index_base < 0 || (long long)index_base + n > (long long)INT_MAX) return fail("index range overflows int");
    qmv::ArgmaxOut am{(unsigned long long *)key, workspace, index_base};
    QMV_CUDA(qmv::launch_argmax(logits, n, am, (cudaStream_t)stream), "argmax launch");
    return 1;
}

QMV_EXPORT int qmv_matvec_argmax(const QmvWeight *w, const float *x, int x_count, float *logits,
                                 int y_count, uint64_t *key, void *workspace, void *stream)
{
    if (!check_weight(w)) return 0;
    if (x == nullptr || logits == nullptr || key == nullptr || workspace == nullptr)
        return fail("x, logits, key or workspace is null");
    if (x_count != w->L.cols || y_count != w->L.rows)
        return fail("counts (%d, %d) do not match the %d x %d weight", x_count, y_count, w->L.rows, w->L.cols);
    if (!aligned16(x)) return fail("x must be 16-byte aligned");
    qmv::ArgmaxOut am{(unsigned long long *)key, workspace, w->row_begin};
    QMV_CUDA(qmv::launch_gemv(w->L, w->dev, x, logits, &am, (cudaStream_t)stream), "gemv+argmax launch");
    return 1;
}

QMV_EXPORT int qmv_argmax_noalloc(const float *logits, int n, int index_base, uint64_t *key, void *stream)
{
    if (logits == nullptr || key == nullptr) return fail("logits or key is null");
    if (n <= 0) return fail("vocabulary size must be positive");
    if (n > qmv::noalloc_max_logits())
        return fail("qmv_argmax_noalloc takes at most %d logits (its static scratch holds one key per "
                    "%d logits); use qmv_argmax with a workspace for %d",
                    qmv::noalloc_max_logits(), qmv::noalloc_max_logits() / 2048, n);
    if (index_base < 0 || (long long)index_base + n > (long long)INT_MAX) return fail("index range overflows int");
    QMV_CUDA(qmv::launch_argmax_noalloc(logits, n, index_base, (unsigned long long *)key, (cudaStream_t)stream),
             "argmax (no allocation) launch");
    return 1;
}

QMV_EXPORT int qmv_exchange_bytes(int world, int slot_rows, size_t *bytes)
{
    if (bytes == nullptr) return fail("bytes pointer is null");
    if (world < 2 || world > qmv::kMaxPeers) return fail("world must be 2..%d", qmv::kMaxPeers);
    if (slot_rows <= 0) return fail("slot_rows must be positive");
    *bytes = qmv::kExchangeHeader + 2 * qmv::exchange_parity_bytes(world, slot_rows);
    return 1;
}

QMV_EXPORT int qmv_ipc_alloc(size_t bytes, void **dev_ptr, void *handle)
{
    if (dev_ptr == nullptr || handle == nullptr || bytes == 0) return fail("bad arguments");
    *dev_ptr = nullptr;
    void *p = nullptr;
    QMV_CUDA(cudaMalloc(&p, bytes), "cudaMalloc(exchange buffer)");
    cudaError_t e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail("exchange buffer", e);
    }
    memcpy(handle, &h, sizeof h);
    *dev_ptr = p;
    return 1;
}

QMV_EXPORT int qmv_ipc_open(const void *handle, void **dev_ptr)
{
    if (dev_ptr == nullptr || handle == nullptr) return fail("bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    QMV_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    return 1;
}

QMV_EXPORT int qmv_ipc_close(void *dev_ptr)
{
    QMV_CUDA(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
    return 1;
}

QMV_EXPORT int qmv_ipc_free(void *dev_ptr)
{
    QMV_CUDA(cudaFree(dev_ptr), "cudaFree(exchange buffer)");
    return 1;
}

QMV_EXPORT int qmv_memcpy(void *dst, const void *src, size_t bytes, void *stream)
{
    if ((dst == nullptr || src == nullptr) && bytes) return fail("dst or src is null");
    QMV_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, (cudaStream_t)stream), "cudaMemcpyAsync");
    QMV_CUDA(cudaStreamSynchronize((cudaStream_t)stream), "cudaStreamSynchronize");
    return 1;
}

QMV_EXPORT int qmv_exchange_logits(void *buffer, int world, int slot_rows, uint32_t epoch, float **logits)
{
    if (buffer == nullptr || logits == nullptr) return fail("bad arguments");
    if (world < 2 || world > qmv::kMaxPeers || slot_rows <= 0) return fail("bad world or slot_rows");
    *logits = (float *)((uint8_t *)buffer + qmv::kExchangeHeader +
                        (epoch & 1u) * qmv::exchange_parity_bytes(world, slot_rows));
    return 1;
}

QMV_EXPORT int qmv_matvec_argmax_exchange(const QmvWeight *w, const float *x, int x_count, int rank, int world,
                                          void *const *buffers, int slot_rows, uint64_t *key, void *workspace,
                                          void *stream)
{
    if (!check_weight(w)) return 0;
    if (x == nullptr || key == nullptr || workspace == nullptr || buffers == nullptr)
        return fail("x, key, workspace or buffers is null");
    if (world < 2 || world > qmv::kMaxPeers) return fail("world must be 2..%d", qmv::kMaxPeers);
    if (rank < 0 || rank >= world) return fail("rank %d outside 0..%d", rank, world - 1);
    if (x_count != w->L.cols) return fail("x_count %d does not match %d columns", x_count, w->L.cols);
    if (slot_rows < w->L.rows || w->row_begin != rank * slot_rows)
        return fail("weight rows [%d, %d) are not rank %d's slot of %d rows", w->row_begin,
                    w->row_begin + w->L.rows, rank, slot_rows);
    if (!aligned16(x)) return fail("x must be 16-byte aligned");
    const size_t pb = qmv::exchange_parity_bytes(world, slot_rows);
    const size_t keys_off = ((size_t)world * slot_rows * 4 + 255) & ~(size_t)255;
    qmv::Exchange ex{};
    ex.world = world;
    ex.rank = rank;
    ex.slot_rows = slot_rows;
    if (buffers[rank] == nullptr) return fail("buffer of rank %d is null", rank);
    ex.epoch = (unsigned int *)buffers[rank];
    const size_t flags_off = keys_off + (size_t)world * qmv::kMaxExCtas * 8;
    for (int p = 0; p < world; ++p) {
        if (buffers[p] == nullptr) return fail("buffer of rank %d is null", p);
        for (int par = 0; par < 2; ++par) {
            uint8_t *base = (uint8_t *)buffers[p] + qmv::kExchangeHeader + par * pb;
            ex.logits[par][p] = (float *)base;
            ex.keys[par][p] = (unsigned long long *)(base + keys_off);
            ex.flags[par][p] = (unsigned int *)(base + flags_off);
        }
    }
    qmv::ArgmaxOut am{(unsigned long long *)key, workspace, w->row_begin};
    QMV_CUDA(qmv::launch_gemv_exchange(w->L, w->dev, x, nullptr, am, ex, (cudaStream_t)stream),
             "gemv+argmax+exchange launch");
    return 1;
}

QMV_EXPORT int qmv_key_to_token(uint64_t key, int *token_id)
{
    if (token_id == nullptr) return fail("token_id is null");
    if (!decode_key(key, token_id)) return fail("argmax saw a non-finite logit");
    return 1;
}

QMV_EXPORT int qmv_greedy_sample(const float *logits, int vocab_size, int *token_id, char *error,
                                 int error_capacity, void *stream)
{
    // Contract of sampler_greedy_sample (src/sampler.cpp:14-36).
    auto set_err = [&](const char *msg) {
        if (error != nullptr && error_capacity > 0) snprintf(error, (size_t)error_capacity, "%s", msg);
        fail("%s", msg);
    };
    if (token_id != nullptr) *token_id = -1;
    if (logits == nullptr || vocab_size <= 0 || token_id == nullptr) {
        set_err("Greedy sampler arguments are invalid.");
        return 0;
    }
    Staging *st = nullptr;
    if (!staging(&st)) {
        set_err(g_error.c_str());
        return 0;
    }
    cudaStream_t s = stream ? (cudaStream_t)stream : st->stream;
    qmv::ArgmaxOut am{st->dkey, st->ws, 0};
    cudaError_t e = qmv::launch_argmax(logits, vocab_size, am, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(st->hkey, st->dkey, sizeof(unsigned long long), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        cuda_fail("greedy sample", e);
        std::string m = g_error;
        set_err(m.c_str());
        return 0;
    }
    int id = -1;
    if (!decode_key(*st->hkey, &id)) {
        set_err("Greedy sampler received a non-finite logit.");
        return 0;
    }
    *token_id = id;
    if (error != nullptr && error_capacity > 0) error[0] = '\0';
    return 1;
}

// Host-pointer drop-in (src/quantized_matvec.h:32-50 contract).
QMV_EXPORT int qmv_quantized_tensor_matvec_f32(const GgufQuantizedTensorView *matrix, const float *input,
                                               int input_count, float *output, int output_count)
{
    if (matrix == nullptr || matrix->data == nullptr || input == nullptr || output == nullptr ||
        input_count <= 0 || output_count <= 0)
        return fail("null pointer or non-positive count");
    int rows = 0, cols = 0;
    if (!check_view(matrix, &rows, &cols)) return 0;
    if (input_count != cols || output_count != rows)
        return fail("input_count/output_count do not match the %d x %d matrix", rows, cols);
    QmvWeight *w = nullptr;
    if (!qmv_resident_weight(matrix, &w)) return 0;
    Staging *st = nullptr;
    if (!staging(&st)) return 0;
    cudaStream_t s = st->stream;
    if (!grow(&st->dx, &st->dx_cap, (size_t)cols, s) || !grow(&st->dy, &st->dy_cap, (size_t)rows, s)) return 0;
    const CallStatus cs(st);
    QMV_CUDA(cudaMemcpyAsync(st->dx, input, sizeof(float) * cols, cudaMemcpyHostToDevice, s), "copy input");
    if (!kernels_begin(st)) return 0;
    QMV_CUDA(qmv::launch_gemv(w->L, w->dev, st->dx, st->dy, nullptr, s), "gemv launch");
    if (!kernels_end(st)) return 0;
    QMV_CUDA(cudaMemcpyAsync(output, st->dy, sizeof(float) * rows, cudaMemcpyDeviceToHost, s), "copy output");
    QMV_CUDA(cudaStreamSynchronize(s), "matvec");
    if (!cs.check("matvec")) return 0;
    return kernels_elapsed(st);
}

QMV_EXPORT int qmv_quantized_tensor_matmul_f32(const GgufQuantizedTensorView *matrix, const float *inputs,
                                               int input_count, int batch_count, float *outputs,
                                               int output_count)
{
    if (matrix == nullptr || matrix->data == nullptr || inputs == nullptr || outputs == nullptr ||
        input_count <= 0 || output_count <= 0 || batch_count <= 0)
        return fail("null pointer or non-positive count");
    int rows = 0, cols = 0;
    if (!check_view(matrix, &rows, &cols)) return 0;
    if (input_count != cols || output_count != rows)
        return fail("input_count/output_count do not match the %d x %d matrix", rows, cols);
    if ((size_t)batch_count > SIZE_MAX / (size_t)input_count ||
        (size_t)batch_count > SIZE_MAX / (size_t)output_count)
        return fail("batch size overflows");
    QmvWeight *w = nullptr;
    if (!qmv_resident_weight(matrix, &w)) return 0;
    Staging *st = nullptr;
    if (!staging(&st)) return 0;
    const size_t nx = (size_t)batch_count * cols, ny = (size_t)batch_count * rows;
    cudaStream_t s = st->stream;
    if (!grow(&st->dx, &st->dx_cap, nx, s) || !grow(&st->dy, &st->dy_cap, ny, s)) return 0;
    const CallStatus cs(st);
    QMV_CUDA(cudaMemcpyAsync(st->dx, inputs, sizeof(float) * nx, cudaMemcpyHostToDevice, s), "copy inputs");
    if (!kernels_begin(st)) return 0;
    QMV_CUDA(qmv::launch_matmul(w->L, w->dev, st->dx, batch_count, st->dy, s), "matmul launch");
    if (!kernels_end(st)) return 0;
    QMV_CUDA(cudaMemcpyAsync(outputs, st->dy, sizeof(float) * ny, cudaMemcpyDeviceToHost, s), "copy outputs");
    QMV_CUDA(cudaStreamSynchronize(s), "matmul");
    if (!cs.check("matmul")) return 0;
    return kernels_elapsed(st);
}
