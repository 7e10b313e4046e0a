// runtime.cu -- lifecycle, errors, memory, transfers, streams and events of
// the C ABI (include/mfcuda.h).  These are the device halves of manifesto's
// tensor.Backend (tensor/backend.go:18-68): Upload/Download become an
// allocation plus an async copy on a caller stream, Close becomes
// mf_shutdown, and Tensor.Sync reads the sticky device status.
#include "mf_runtime.h"

#include <cstring>
#include <mutex>
#include <string>

namespace mf {

namespace {
thread_local std::string t_last_error;
DeviceState g_state;
std::mutex g_init_mutex;
}  // namespace

__device__ int g_sticky_status = 0;

int* sticky_status_ptr() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sticky_status) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return static_cast<int*>(p);
}

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(MF_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

DeviceState& state() { return g_state; }

int enter() {
    if (!g_state.open) return fail(MF_ERR_BACKEND_CLOSED, "mfcuda: backend not initialised (call mf_init)");
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != g_state.device) {
        cudaError_t err = cudaSetDevice(g_state.device);
        if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
    }
    return MF_OK;
}

int64_t stream_grid(int64_t work_items, int threads, int blocks_per_sm) {
    const int64_t per_block = threads;
    int64_t blocks = (work_items + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(g_state.sm_count > 0 ? g_state.sm_count : 148) * blocks_per_sm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return blocks;
}

// One thread polls the flag with acquire loads, sleeping between polls; when
// the poll budget runs out it records MF_DEVICE_TIMEOUT and returns, so the
// stream moves on and the context stays usable.
__global__ void wait_flag_kernel(const int* flag, int expect, int64_t max_polls, int* status) {
    for (int64_t i = 0; i < max_polls; ++i) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v == expect) return;
        __nanosleep(256);
    }
    atomicExch(status, MF_DEVICE_TIMEOUT);
}

}  // namespace mf

using namespace mf;

extern "C" {

int mf_abi_version(void) { return MFCUDA_ABI_VERSION; }

int mf_device_count(int* count) {
    if (!count) return fail(MF_ERR_INVALID_ARGUMENT, "mf_device_count: count is NULL");
    int c = 0;
    cudaError_t err = cudaGetDeviceCount(&c);
    if (err != cudaSuccess) {
        cudaGetLastError();  // clear: no driver / no device simply means zero devices
        c = 0;
    }
    *count = c;
    return MF_OK;
}

int mf_init(int device) {
    std::lock_guard<std::mutex> lock(g_init_mutex);
    int count = 0;
    cudaError_t err = cudaGetDeviceCount(&count);
    if (err != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(MF_ERR_NEEDS_PLATFORM_SETUP, "mf_init: no CUDA device available (%s)",
                    err == cudaSuccess ? "device count 0" : cudaGetErrorString(err));
    }
    if (device < 0 || device >= count)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_init: device %d out of range [0,%d)", device, count);
    MF_CUDA_CHECK(cudaSetDevice(device));
    cudaDeviceProp prop;
    MF_CUDA_CHECK(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10)
        return fail(MF_ERR_NEEDS_PLATFORM_SETUP,
                    "mf_init: device %d is sm_%d%d; this library is built for sm_100a only",
                    device, prop.major, prop.minor);
    MF_CUDA_CHECK(cudaFree(nullptr));  // create the primary context now
    g_state.device = device;
    g_state.sm_count = prop.multiProcessorCount;
    g_state.max_threads_per_sm = prop.maxThreadsPerMultiProcessor;
    g_state.open = true;
    return MF_OK;
}

int mf_shutdown(void) {
    std::lock_guard<std::mutex> lock(g_init_mutex);
    if (!g_state.open) return MF_OK;
    cudaSetDevice(g_state.device);
    cudaError_t err = cudaDeviceSynchronize();
    g_state.open = false;
    if (err != cudaSuccess) return cuda_fail(err, "mf_shutdown: cudaDeviceSynchronize");
    return MF_OK;
}

const char* mf_last_error(void) { return t_last_error.c_str(); }

int mf_last_error_copy(char* buf, size_t n) {
    if (!buf || n == 0) return fail(MF_ERR_INVALID_ARGUMENT, "mf_last_error_copy: empty buffer");
    std::strncpy(buf, t_last_error.c_str(), n - 1);
    buf[n - 1] = '\0';
    return MF_OK;
}

int mf_device_status(int* device_code) {
    MF_ENTER();
    MF_CUDA_CHECK(cudaDeviceSynchronize());
    int code = 0;
    MF_CUDA_CHECK(cudaMemcpyFromSymbol(&code, g_sticky_status, sizeof(int)));
    if (device_code) *device_code = code;
    if (code != 0) {
        const int zero = 0;
        MF_CUDA_CHECK(cudaMemcpyToSymbol(g_sticky_status, &zero, sizeof(int)));
        return fail(MF_ERR_DEVICE_STICKY, "mfcuda: a kernel recorded device status %d", code);
    }
    return MF_OK;
}

int mf_wait_flag(const int* flag, int expect, int64_t max_polls, mf_stream stream) {
    MF_ENTER();
    if (!flag) return fail(MF_ERR_INVALID_ARGUMENT, "mf_wait_flag: flag is NULL");
    if (reinterpret_cast<uintptr_t>(flag) % alignof(int))
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_wait_flag: flag is not 4-byte aligned");
    if (max_polls < 0) return fail(MF_ERR_INVALID_ARGUMENT, "mf_wait_flag: negative poll budget");
    int* status = sticky_status_ptr();
    if (!status) return fail(MF_ERR_CUDA, "mf_wait_flag: sticky status word unavailable");
    wait_flag_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flag, expect, max_polls, status);
    MF_LAUNCH_CHECK("mf_wait_flag");
    return MF_OK;
}

int mf_device_info(int* sm_count, int* cc_major, int* cc_minor, size_t* total_bytes) {
    MF_ENTER();
    cudaDeviceProp prop;
    MF_CUDA_CHECK(cudaGetDeviceProperties(&prop, g_state.device));
    if (sm_count) *sm_count = prop.multiProcessorCount;
    if (cc_major) *cc_major = prop.major;
    if (cc_minor) *cc_minor = prop.minor;
    if (total_bytes) *total_bytes = prop.totalGlobalMem;
    return MF_OK;
}

int mf_alloc(void** dptr, size_t bytes) {
    MF_ENTER();
    if (!dptr) return fail(MF_ERR_INVALID_ARGUMENT, "mf_alloc: dptr is NULL");
    *dptr = nullptr;
    if (bytes == 0) return MF_OK;
    cudaError_t err = cudaMalloc(dptr, bytes);
    if (err == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return fail(MF_ERR_ALLOCATOR_EXHAUSTED, "mf_alloc: %zu bytes: out of device memory", bytes);
    }
    if (err != cudaSuccess) return cuda_fail(err, "cudaMalloc");
    return MF_OK;
}

int mf_free(void* dptr) {
    MF_ENTER();
    if (!dptr) return MF_OK;
    MF_CUDA_CHECK(cudaFree(dptr));
    return MF_OK;
}

int mf_host_alloc(void** hptr, size_t bytes) {
    MF_ENTER();
    if (!hptr) return fail(MF_ERR_INVALID_ARGUMENT, "mf_host_alloc: hptr is NULL");
    *hptr = nullptr;
    if (bytes == 0) return MF_OK;
    cudaError_t err = cudaMallocHost(hptr, bytes);
    if (err == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return fail(MF_ERR_ALLOCATOR_EXHAUSTED, "mf_host_alloc: %zu bytes: out of pinned memory", bytes);
    }
    if (err != cudaSuccess) return cuda_fail(err, "cudaMallocHost");
    return MF_OK;
}

int mf_host_free(void* hptr) {
    MF_ENTER();
    if (!hptr) return MF_OK;
    MF_CUDA_CHECK(cudaFreeHost(hptr));
    return MF_OK;
}

static int copy_async(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, mf_stream stream,
                      const char* name) {
    MF_ENTER();
    if (bytes == 0) return MF_OK;
    if (!dst || !src) return fail(MF_ERR_INVALID_ARGUMENT, "%s: NULL pointer", name);
    cudaError_t err = cudaMemcpyAsync(dst, src, bytes, kind, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, name);
    return MF_OK;
}

int mf_memcpy_h2d_async(void* dst, const void* src, size_t bytes, mf_stream stream) {
    return copy_async(dst, src, bytes, cudaMemcpyHostToDevice, stream, "mf_memcpy_h2d_async");
}
int mf_memcpy_d2h_async(void* dst, const void* src, size_t bytes, mf_stream stream) {
    return copy_async(dst, src, bytes, cudaMemcpyDeviceToHost, stream, "mf_memcpy_d2h_async");
}
int mf_memcpy_d2d_async(void* dst, const void* src, size_t bytes, mf_stream stream) {
    return copy_async(dst, src, bytes, cudaMemcpyDeviceToDevice, stream, "mf_memcpy_d2d_async");
}

int mf_memset_async(void* dst, int value, size_t bytes, mf_stream stream) {
    MF_ENTER();
    if (bytes == 0) return MF_OK;
    if (!dst) return fail(MF_ERR_INVALID_ARGUMENT, "mf_memset_async: NULL pointer");
    MF_CUDA_CHECK(cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream)));
    return MF_OK;
}

int mf_stream_create(mf_stream* stream) {
    MF_ENTER();
    if (!stream) return fail(MF_ERR_INVALID_ARGUMENT, "mf_stream_create: NULL out pointer");
    cudaStream_t s;
    MF_CUDA_CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *stream = s;
    return MF_OK;
}

int mf_stream_destroy(mf_stream stream) {
    MF_ENTER();
    if (!stream) return MF_OK;
    MF_CUDA_CHECK(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
    return MF_OK;
}

int mf_stream_sync(mf_stream stream) {
    MF_ENTER();
    MF_CUDA_CHECK(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    return MF_OK;
}

int mf_event_create(mf_event* event, int enable_timing) {
    MF_ENTER();
    if (!event) return fail(MF_ERR_INVALID_ARGUMENT, "mf_event_create: NULL out pointer");
    cudaEvent_t e;
    MF_CUDA_CHECK(cudaEventCreateWithFlags(&e, enable_timing ? cudaEventDefault : cudaEventDisableTiming));
    *event = e;
    return MF_OK;
}

int mf_event_destroy(mf_event event) {
    MF_ENTER();
    if (!event) return MF_OK;
    MF_CUDA_CHECK(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
    return MF_OK;
}

int mf_event_record(mf_event event, mf_stream stream) {
    MF_ENTER();
    if (!event) return fail(MF_ERR_INVALID_ARGUMENT, "mf_event_record: NULL event");
    MF_CUDA_CHECK(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
    return MF_OK;
}

int mf_stream_wait_event(mf_stream stream, mf_event event) {
    MF_ENTER();
    if (!event) return fail(MF_ERR_INVALID_ARGUMENT, "mf_stream_wait_event: NULL event");
    MF_CUDA_CHECK(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0));
    return MF_OK;
}

int mf_event_sync(mf_event event) {
    MF_ENTER();
    if (!event) return fail(MF_ERR_INVALID_ARGUMENT, "mf_event_sync: NULL event");
    MF_CUDA_CHECK(cudaEventSynchronize(static_cast<cudaEvent_t>(event)));
    return MF_OK;
}

int mf_event_elapsed_ms(mf_event start, mf_event stop, float* ms) {
    MF_ENTER();
    if (!start || !stop || !ms) return fail(MF_ERR_INVALID_ARGUMENT, "mf_event_elapsed_ms: NULL argument");
    MF_CUDA_CHECK(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(stop)));
    return MF_OK;
}

int mf_device_sync(void) {
    MF_ENTER();
    MF_CUDA_CHECK(cudaDeviceSynchronize());
    return MF_OK;
}

}  // extern "C"
