// SPDX-License-Identifier: Unlicense
//
// Device runtime: the roles of the reference's ocl_backend.c (device
// pick, buffers, blocking transfers, fatal errors) on CUDA, plus the
// error-recording mode and the per-launch profiler of ops_report
// (the reference's ops_run / ops_report, ops.c:25-67).

#include <ctype.h>
#include <mutex>
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>
#include <string>
#include <vector>

#include "common.cuh"

// ------------------------------------------------------------------ errors

static int g_error_mode = COREG_ERRORS_FATAL;
static thread_local std::string t_error;
static thread_local bool t_has_error = false;

extern "C" void coreg_set_error_mode(int mode) { g_error_mode = mode; }

extern "C" const char *coreg_last_error(void)
{
    return t_has_error ? t_error.c_str() : NULL;
}

extern "C" void coreg_clear_error(void)
{
    t_has_error = false;
    t_error.clear();
}

namespace coreg {

void fail(const char *fmt, ...)
{
    char buf[1024];
    va_list ap;

    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (g_error_mode == COREG_ERRORS_FATAL) {
        fprintf(stderr, "ERROR: %s\n", buf);
        fflush(stderr);
        exit(1);
    }
    if (!t_has_error) {
        t_has_error = true;
        t_error = buf;
    }
}

bool pending() { return t_has_error; }

bool cuda_ok(cudaError_t e, const char *what)
{
    if (e == cudaSuccess)
        return true;
    fail("CUDA: %s failed: %s", what, cudaGetErrorString(e));
    return false;
}

bool launch_ok(const char *what)
{
    return cuda_ok(cudaGetLastError(), what);
}

bool count_ok(long n, const char *what)
{
    if (n < 0 || n > 0x7fffffffL) {
        fail("CUDA: %s of %ld elements exceeds 2^31", what, n);
        return false;
    }
    return true;
}

// ---------------------------------------------------------------- profiler

struct ProfEntry {
    std::string what;
    double ms;
    long calls;
};
static std::mutex g_prof_mu;
static std::vector<ProfEntry> g_prof;

Prof::Prof(const struct ocl_backend *ocl, const char *w)
    : what(w), st(stream_of(ocl)), on(ocl && ocl->profile)
{
    if (on) {
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, st);
    }
}

Prof::~Prof()
{
    float ms = 0;

    if (!on)
        return;
    cudaEventRecord(e1, st);
    cudaEventSynchronize(e1);
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (auto &p : g_prof)
        if (p.what == what) {
            p.ms += ms;
            p.calls++;
            return;
        }
    g_prof.push_back({what, ms, 1});
}

}  // namespace coreg

extern "C" void ops_report(void)
{
    std::lock_guard<std::mutex> lk(coreg::g_prof_mu);
    for (auto &p : coreg::g_prof)
        fprintf(stderr, "%-24s %10.3f ms %8ld calls\n", p.what.c_str(), p.ms,
                p.calls);
}

// Reset of the profiler totals (no reference counterpart).
extern "C" void ops_report_reset(void)
{
    std::lock_guard<std::mutex> lk(coreg::g_prof_mu);
    coreg::g_prof.clear();
}

// Totals as text lines "name ms calls" into buf (no reference
// counterpart); returns the bytes needed.
extern "C" size_t ops_report_text(char *buf, size_t n)
{
    std::lock_guard<std::mutex> lk(coreg::g_prof_mu);
    std::string s;
    char line[256];

    for (auto &p : coreg::g_prof) {
        snprintf(line, sizeof(line), "%s %.6f %ld\n", p.what.c_str(), p.ms,
                 p.calls);
        s += line;
    }
    if (buf && n) {
        size_t k = s.size() < n - 1 ? s.size() : n - 1;
        memcpy(buf, s.data(), k);
        buf[k] = 0;
    }
    return s.size() + 1;
}

// ----------------------------------------------------------------- backend

using namespace coreg;

extern "C" const char *ocl_errstr(cl_int err)
{
    return cudaGetErrorString((cudaError_t)err);
}

extern "C" void ocl_check(cl_int err, const char *what)
{
    if (err != 0)
        fail("CUDA: %s failed: %s", what, ocl_errstr(err));
}

extern "C" void ocl_init(struct ocl_backend *ocl, const char *device_opt,
                         const char *platform_opt)
{
    int n = 0, dev = 0, rt = 0;
    cudaDeviceProp prop;
    const char *prof;

    (void)platform_opt;
    memset(ocl, 0, sizeof(*ocl));
    if (pending())
        return;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        fail("CUDA: no usable %s device found",
             device_opt ? device_opt : "auto");
        return;
    }
    if (!device_opt || !strcmp(device_opt, "auto") || !strcmp(device_opt, "gpu"))
        cudaGetDevice(&dev);
    else {
        const char *p = device_opt;
        char *end = NULL;
        long v;

        while (*p && isspace((unsigned char)*p))
            p++;
        v = strtol(p, &end, 10);
        if (end == p || *end || v < 0 || v >= n) {
            fail("Invalid device option <%s> (%d CUDA device(s))", device_opt,
                 n);
            return;
        }
        dev = (int)v;
    }
    if (!cuda_ok(cudaSetDevice(dev), "cudaSetDevice"))
        return;
    if (!cuda_ok(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties"))
        return;
    if (prop.major != 10 || prop.minor != 0) {
        fail("CUDA: device %d (%s) is compute capability %d.%d; this build "
             "has kernels for sm_100a only",
             dev, prop.name, prop.major, prop.minor);
        return;
    }
    ocl->device = dev;
    snprintf(ocl->device_name, sizeof(ocl->device_name), "%s", prop.name);
    cudaRuntimeGetVersion(&rt);
    snprintf(ocl->platform_name, sizeof(ocl->platform_name), "CUDA %d.%d",
             rt / 1000, (rt % 1000) / 10);
    ocl->global_mem = prop.totalGlobalMem;
    ocl->max_alloc = prop.totalGlobalMem;
    ocl->is_gpu = 1;
    ocl->sm_count = prop.multiProcessorCount;
    ocl->cc_major = prop.major;
    ocl->cc_minor = prop.minor;
    prof = getenv("I_COREGISTRATION_OPENCL_PROFILE");
    ocl->profile = prof && *prof;
    {
        cudaStream_t st;

        if (!cuda_ok(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking),
                     "cudaStreamCreate"))
            return;
        ocl->queue = st;
    }
}

extern "C" void ocl_free(struct ocl_backend *ocl)
{
    if (ocl->queue) {
        cudaSetDevice(ocl->device);
        cudaStreamSynchronize(stream_of(ocl));
        cudaStreamDestroy(stream_of(ocl));
    }
    if (ocl->pinned)
        cudaFreeHost(ocl->pinned);
    memset(ocl, 0, sizeof(*ocl));
}

extern "C" cl_mem ocl_alloc(struct ocl_backend *ocl, size_t n, const char *what)
{
    void *p = NULL;
    cudaError_t e;
    cl_mem m;

    if (pending())
        return NULL;
    if (n == 0)
        n = 4;
    if (ocl->max_alloc && n > ocl->max_alloc) {
        fail("CUDA: buffer <%s> needs %lu MiB, more than the device memory "
             "of %lu MiB",
             what, (unsigned long)(n >> 20),
             (unsigned long)(ocl->max_alloc >> 20));
        return NULL;
    }
    e = cudaMalloc(&p, n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail("CUDA: allocating %lu MiB for <%s> failed: %s",
             (unsigned long)(n >> 20), what, cudaGetErrorString(e));
        return NULL;
    }
    m = (cl_mem)malloc(sizeof(*m));
    m->ptr = p;
    m->bytes = n;
    m->owned = 1;
    return m;
}

extern "C" cl_mem ocl_wrap(void *dptr, size_t n)
{
    cl_mem m = (cl_mem)malloc(sizeof(*m));

    m->ptr = dptr;
    m->bytes = n;
    m->owned = 0;
    return m;
}

extern "C" void *ocl_ptr(cl_mem m) { return m ? m->ptr : NULL; }
extern "C" size_t ocl_bytes(cl_mem m) { return m ? m->bytes : 0; }

static bool range_ok(cl_mem m, size_t off, size_t n, const char *what)
{
    if (!m) {
        fail("CUDA: %s on a NULL buffer", what);
        return false;
    }
    if (off > m->bytes || n > m->bytes - off) {
        fail("CUDA: %s of %zu bytes at %zu outside a buffer of %zu bytes",
             what, n, off, m->bytes);
        return false;
    }
    return true;
}

// Host buffer: pinned memory is copied directly, pageable memory through
// the backend's pinned staging buffer (in chunks), so that the copy is
// one asynchronous DMA on the stream followed by a wait.
static bool is_pinned(const void *p)
{
    cudaPointerAttributes a;

    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

static const size_t STAGE = (size_t)64 << 20;

static bool stage(struct ocl_backend *ocl)
{
    if (ocl->pinned)
        return true;
    if (!cuda_ok(cudaMallocHost(&ocl->pinned, STAGE), "cudaMallocHost"))
        return false;
    ocl->pinned_bytes = STAGE;
    return true;
}

extern "C" void ocl_write(struct ocl_backend *ocl, cl_mem dst, size_t off,
                          const void *src, size_t n)
{
    cudaStream_t st = stream_of(ocl);

    if (pending() || !range_ok(dst, off, n, "ocl_write"))
        return;
    if (is_pinned(src)) {
        cuda_ok(cudaMemcpyAsync((char *)dst->ptr + off, src, n,
                                cudaMemcpyHostToDevice, st),
                "cudaMemcpyAsync H2D");
        cuda_ok(cudaStreamSynchronize(st), "ocl_write");
        return;
    }
    if (!stage(ocl))
        return;
    for (size_t done = 0; done < n;) {
        size_t k = n - done < STAGE ? n - done : STAGE;

        // The staging buffer is reused: wait for its previous copy.
        if (!cuda_ok(cudaStreamSynchronize(st), "ocl_write"))
            return;
        memcpy(ocl->pinned, (const char *)src + done, k);
        if (!cuda_ok(cudaMemcpyAsync((char *)dst->ptr + off + done, ocl->pinned,
                                     k, cudaMemcpyHostToDevice, st),
                     "cudaMemcpyAsync H2D"))
            return;
        done += k;
    }
    cuda_ok(cudaStreamSynchronize(st), "ocl_write");
}

extern "C" void ocl_read(struct ocl_backend *ocl, cl_mem src, size_t off,
                         void *dst, size_t n)
{
    cudaStream_t st = stream_of(ocl);

    if (pending() || !range_ok(src, off, n, "ocl_read"))
        return;
    if (is_pinned(dst)) {
        cuda_ok(cudaMemcpyAsync(dst, (const char *)src->ptr + off, n,
                                cudaMemcpyDeviceToHost, st),
                "cudaMemcpyAsync D2H");
        cuda_ok(cudaStreamSynchronize(st), "ocl_read");
        return;
    }
    if (!stage(ocl))
        return;
    for (size_t done = 0; done < n;) {
        size_t k = n - done < STAGE ? n - done : STAGE;

        if (!cuda_ok(cudaMemcpyAsync(ocl->pinned,
                                     (const char *)src->ptr + off + done, k,
                                     cudaMemcpyDeviceToHost, st),
                     "cudaMemcpyAsync D2H"))
            return;
        if (!cuda_ok(cudaStreamSynchronize(st), "ocl_read"))
            return;
        memcpy((char *)dst + done, ocl->pinned, k);
        done += k;
    }
}

extern "C" cl_mem ocl_upload(struct ocl_backend *ocl, const void *src, size_t n,
                             const char *what)
{
    cl_mem m = ocl_alloc(ocl, n, what);

    if (m)
        ocl_write(ocl, m, 0, src, n);
    return m;
}

extern "C" void ocl_release(cl_mem *m)
{
    if (!m || !*m)
        return;
    if ((*m)->owned && (*m)->ptr)
        cudaFree((*m)->ptr);
    free(*m);
    *m = NULL;
}

extern "C" void ocl_copy(struct ocl_backend *ocl, cl_mem src, size_t soff,
                         cl_mem dst, size_t doff, size_t n)
{
    if (pending() || !range_ok(src, soff, n, "ocl_copy") ||
        !range_ok(dst, doff, n, "ocl_copy"))
        return;
    cuda_ok(cudaMemcpyAsync((char *)dst->ptr + doff,
                            (const char *)src->ptr + soff, n,
                            cudaMemcpyDeviceToDevice, stream_of(ocl)),
            "cudaMemcpyAsync D2D");
}

extern "C" void ocl_zero(struct ocl_backend *ocl, cl_mem m, size_t off, size_t n)
{
    if (pending() || !range_ok(m, off, n, "ocl_zero"))
        return;
    cuda_ok(cudaMemsetAsync((char *)m->ptr + off, 0, n, stream_of(ocl)),
            "cudaMemsetAsync");
}

extern "C" cl_int clFinish(cl_command_queue queue)
{
    return (cl_int)cudaStreamSynchronize((cudaStream_t)queue);
}

extern "C" void ocl_join(struct ocl_backend *dst, struct ocl_backend *src)
{
    if (pending())
        return;
    if (!dst || !src || dst->device != src->device) {
        fail("ocl_join: backends of different devices");
        return;
    }
    cudaEvent_t ev;
    if (!cuda_ok(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate"))
        return;
    if (cuda_ok(cudaEventRecord(ev, stream_of(src)), "cudaEventRecord"))
        cuda_ok(cudaStreamWaitEvent(stream_of(dst), ev, 0), "cudaStreamWaitEvent");
    cudaEventDestroy(ev);
}

extern "C" void ocl_finish(struct ocl_backend *ocl)
{
    if (pending())
        return;
    cuda_ok(cudaStreamSynchronize(stream_of(ocl)), "cudaStreamSynchronize");
}

// One pair of timing events per thread (ocl_timer_start / _stop).
static thread_local cudaEvent_t t_ev0 = nullptr, t_ev1 = nullptr;

extern "C" void ocl_timer_start(struct ocl_backend *ocl)
{
    if (pending())
        return;
    if (!t_ev0) {
        cudaEventCreate(&t_ev0);
        cudaEventCreate(&t_ev1);
    }
    cuda_ok(cudaEventRecord(t_ev0, stream_of(ocl)), "cudaEventRecord");
}

extern "C" double ocl_timer_stop(struct ocl_backend *ocl)
{
    float ms = 0;
    if (pending() || !t_ev0)
        return -1;
    if (!cuda_ok(cudaEventRecord(t_ev1, stream_of(ocl)), "cudaEventRecord") ||
        !cuda_ok(cudaEventSynchronize(t_ev1), "cudaEventSynchronize") ||
        !cuda_ok(cudaEventElapsedTime(&ms, t_ev0, t_ev1), "cudaEventElapsedTime"))
        return -1;
    return ms;
}
