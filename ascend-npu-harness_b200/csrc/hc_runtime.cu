// C-ABI device runtime shim over the CUDA runtime (declared in include/hc_runtime.h).
//
// Replaces the reference's dlopen-based Ascend runtime (src/ascend_runtime.cpp:52-243):
// same operations, real device events instead of the reference's stubs
// (src/ascend_runtime.cpp:238-243), per-thread current device, and int status codes.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "hc_internal.h"

namespace hc {

namespace {

thread_local int t_last_status = HC_OK;
thread_local char t_last_msg[512] = "";

// ---- fault injection ------------------------------------------------------------------
std::mutex g_fault_mu;
std::string g_fault_kind;
long g_fault_target = 0;
std::atomic<long> g_fault_count{0};
bool g_fault_env_read = false;

void parse_fault(const char* spec) {
    g_fault_kind.clear();
    g_fault_target = 0;
    g_fault_count.store(0);
    if (!spec || !*spec) return;
    const char* colon = std::strchr(spec, ':');
    if (!colon) return;
    g_fault_kind.assign(spec, colon - spec);
    g_fault_target = std::strtol(colon + 1, nullptr, 10);
}

// ---- device error words ------------------------------------------------------------------
std::mutex g_words_mu;
std::vector<error_word_reader>& error_readers() {
    static std::vector<error_word_reader> v;
    return v;
}

}  // namespace

int fail(int status, const char* fmt, ...) {
    t_last_status = status;
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(t_last_msg, sizeof(t_last_msg), fmt, ap);
    va_end(ap);
    return status;
}

int ok() {
    t_last_status = HC_OK;
    t_last_msg[0] = '\0';
    return HC_OK;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(HC_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

bool fault_hit(const char* kind) {
    {
        std::lock_guard<std::mutex> lk(g_fault_mu);
        if (!g_fault_env_read) {
            g_fault_env_read = true;
            parse_fault(std::getenv("HC_FAULT"));
        }
        if (g_fault_kind.empty() || g_fault_kind != kind) return false;
    }
    long n = g_fault_count.fetch_add(1) + 1;
    return n == g_fault_target;
}

int resident_blocks(const void* kernel, int threads, size_t smem) {
    struct Entry {
        const void* kernel;
        int threads, dev;
        size_t smem;
        int blocks;
    };
    static std::mutex mu;
    static std::vector<Entry> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Entry& e : cache)
            if (e.kernel == kernel && e.threads == threads && e.smem == smem && e.dev == dev) return e.blocks;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm <= 0) {
        cudaGetLastError();  // a failed query leaves its error pending; clear it
        per_sm = 1;
    }
    const int blocks = per_sm * sm_count();
    std::lock_guard<std::mutex> lock(mu);
    cache.push_back(Entry{kernel, threads, dev, smem, blocks});
    return blocks;
}

int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int sms = cache[dev].load(std::memory_order_relaxed);
    if (sms == 0) {
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
            sms = 148;
        cache[dev].store(sms, std::memory_order_relaxed);
    }
    return sms;
}

uint64_t current_context_id() {
    using GetCurrentFn = int (*)(void**);
    using GetIdFn = int (*)(void*, unsigned long long*);
    static std::once_flag once;
    static GetCurrentFn get_current = nullptr;
    static GetIdFn get_id = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrentFn>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetIdFn>(p);
        cudaGetLastError();
    });
    if (!get_current || !get_id) return 0;
    void* ctx = nullptr;  // none until the runtime has bound the device's primary context to the thread
    unsigned long long id = 0;
    if (get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
    return static_cast<uint64_t>(id);
}

int set_max_dynamic_smem(const void* kernel, size_t bytes, const char* name) {
    struct Entry {
        const void* kernel;
        int dev;
        size_t bytes;
    };
    static std::mutex mu;
    static std::vector<Entry> done;
    int dev = 0;
    HC_CHECK_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry& e : done)
        if (e.kernel == kernel && e.dev == dev && e.bytes >= bytes) return HC_OK;
    const cudaError_t err =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(HC_ERR_CUDA, "cudaFuncSetAttribute(%s, %zu B) on device %d: %s", name, bytes, dev,
                    cudaGetErrorString(err));
    }
    for (Entry& e : done)
        if (e.kernel == kernel && e.dev == dev) {
            e.bytes = bytes;
            return HC_OK;
        }
    done.push_back(Entry{kernel, dev, bytes});
    return HC_OK;
}

size_t dtype_size(int dtype) {
    switch (dtype) {
        case HC_DTYPE_F32: return 4;
        case HC_DTYPE_F16: return 2;
        case HC_DTYPE_BF16: return 2;
        case HC_DTYPE_I32: return 4;
        case HC_DTYPE_I8: return 1;
        case HC_DTYPE_U8: return 1;
        default: return 0;
    }
}

int check_launch(const char* kernel) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail(HC_ERR_CUDA, "launch of %s failed: %s", kernel, cudaGetErrorString(err));
    return ok();
}

void register_error_word(error_word_reader reader) {
    std::lock_guard<std::mutex> lk(g_words_mu);
    for (auto r : error_readers())
        if (r == reader) return;
    error_readers().push_back(reader);
}

}  // namespace hc

using hc::cuda_fail;
using hc::fail;
using hc::ok;

extern "C" {

int hc_init(void) {
    int n = 0;
    cudaError_t err = cudaGetDeviceCount(&n);
    if (err != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(HC_ERR_NO_DEVICE, "no CUDA device: %s", err == cudaSuccess ? "count is 0" : cudaGetErrorString(err));
    }
    HC_CHECK_CUDA(cudaFree(nullptr));  // creates the primary context of the current device
    return ok();
}

int hc_device_count(int* count) {
    if (!count) return fail(HC_ERR_INVALID, "hc_device_count: null count");
    int n = 0;
    cudaError_t err = cudaGetDeviceCount(&n);
    if (err != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        return fail(HC_ERR_NO_DEVICE, "cudaGetDeviceCount: %s", cudaGetErrorString(err));
    }
    *count = n;
    if (n == 0) return fail(HC_ERR_NO_DEVICE, "no CUDA device visible");
    return ok();
}

int hc_set_device(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return fail(HC_ERR_INVALID, "hc_set_device(%d): %d device(s) visible", device, n);
    }
    HC_CHECK_CUDA(cudaSetDevice(device));
    return ok();
}

int hc_get_device(int* device) {
    if (!device) return fail(HC_ERR_INVALID, "hc_get_device: null");
    HC_CHECK_CUDA(cudaGetDevice(device));
    return ok();
}

int hc_driver_version(int* version) {
    if (!version) return fail(HC_ERR_INVALID, "hc_driver_version: null");
    HC_CHECK_CUDA(cudaDriverGetVersion(version));
    return ok();
}

int hc_device_sm_count(int* sms) {
    if (!sms) return fail(HC_ERR_INVALID, "hc_device_sm_count: null");
    int dev = 0;
    HC_CHECK_CUDA(cudaGetDevice(&dev));
    HC_CHECK_CUDA(cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev));
    return ok();
}

int hc_device_name(char* buf, size_t buflen) {
    if (!buf || buflen == 0) return fail(HC_ERR_INVALID, "hc_device_name: empty buffer");
    int dev = 0;
    HC_CHECK_CUDA(cudaGetDevice(&dev));
    cudaDeviceProp prop;
    HC_CHECK_CUDA(cudaGetDeviceProperties(&prop, dev));
    std::snprintf(buf, buflen, "%s (sm_%d%d)", prop.name, prop.major, prop.minor);
    return ok();
}

int hc_malloc(void** ptr, size_t bytes) {
    if (!ptr || bytes == 0) return fail(HC_ERR_INVALID, "hc_malloc: null out-pointer or zero size");
    *ptr = nullptr;
    if (hc::fault_hit("malloc")) return fail(HC_ERR_INJECTED, "hc_malloc: injected failure");
    HC_CHECK_CUDA(cudaMalloc(ptr, bytes));
    return ok();
}

int hc_free(void* ptr) {
    if (!ptr) return ok();
    HC_CHECK_CUDA(cudaFree(ptr));
    return ok();
}

int hc_malloc_host(void** ptr, size_t bytes) {
    if (!ptr || bytes == 0) return fail(HC_ERR_INVALID, "hc_malloc_host: null out-pointer or zero size");
    *ptr = nullptr;
    if (hc::fault_hit("malloc")) return fail(HC_ERR_INJECTED, "hc_malloc_host: injected failure");
    HC_CHECK_CUDA(cudaMallocHost(ptr, bytes));
    return ok();
}

int hc_free_host(void* ptr) {
    if (!ptr) return ok();
    HC_CHECK_CUDA(cudaFreeHost(ptr));
    return ok();
}

static int memcpy_impl(void* dst, const void* src, size_t bytes, void* stream, cudaMemcpyKind kind,
                       const char* name) {
    if (bytes == 0) return ok();
    if (!dst || !src) return fail(HC_ERR_INVALID, "%s: null pointer", name);
    if (hc::fault_hit("memcpy")) return fail(HC_ERR_INJECTED, "%s: injected failure", name);
    if (stream == nullptr) {
        HC_CHECK_CUDA(cudaMemcpy(dst, src, bytes, kind));
    } else {
        HC_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, kind, static_cast<cudaStream_t>(stream)));
    }
    return ok();
}

int hc_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
    return memcpy_impl(dst, src, bytes, stream, cudaMemcpyHostToDevice, "hc_memcpy_h2d");
}

int hc_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
    return memcpy_impl(dst, src, bytes, stream, cudaMemcpyDeviceToHost, "hc_memcpy_d2h");
}

int hc_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
    return memcpy_impl(dst, src, bytes, stream, cudaMemcpyDeviceToDevice, "hc_memcpy_d2d");
}

int hc_memset(void* dst, int value, size_t bytes, void* stream) {
    if (bytes == 0) return ok();
    if (!dst) return fail(HC_ERR_INVALID, "hc_memset: null pointer");
    HC_CHECK_CUDA(cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream)));
    if (stream == nullptr) HC_CHECK_CUDA(cudaStreamSynchronize(nullptr));
    return ok();
}

int hc_stream_create(void** stream) {
    if (!stream) return fail(HC_ERR_INVALID, "hc_stream_create: null");
    cudaStream_t s = nullptr;
    HC_CHECK_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *stream = s;
    return ok();
}

int hc_stream_destroy(void* stream) {
    if (!stream) return ok();
    HC_CHECK_CUDA(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
    return ok();
}

int hc_stream_sync(void* stream) {
    HC_CHECK_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    return ok();
}

int hc_device_sync(void) {
    HC_CHECK_CUDA(cudaDeviceSynchronize());
    return ok();
}

int hc_event_create(void** event) {
    if (!event) return fail(HC_ERR_INVALID, "hc_event_create: null");
    cudaEvent_t e = nullptr;
    HC_CHECK_CUDA(cudaEventCreate(&e));
    *event = e;
    return ok();
}

int hc_event_destroy(void* event) {
    if (!event) return ok();
    HC_CHECK_CUDA(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
    return ok();
}

int hc_event_record(void* event, void* stream) {
    if (!event) return fail(HC_ERR_INVALID, "hc_event_record: null event");
    HC_CHECK_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
    return ok();
}

int hc_event_sync(void* event) {
    if (!event) return fail(HC_ERR_INVALID, "hc_event_sync: null event");
    HC_CHECK_CUDA(cudaEventSynchronize(static_cast<cudaEvent_t>(event)));
    return ok();
}

int hc_event_elapsed_ms(float* ms, void* start_event, void* end_event) {
    if (!ms || !start_event || !end_event) return fail(HC_ERR_INVALID, "hc_event_elapsed_ms: null argument");
    HC_CHECK_CUDA(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start_event), static_cast<cudaEvent_t>(end_event)));
    return ok();
}

int hc_check_device_error(void) {
    std::vector<hc::error_word_reader> readers;
    {
        std::lock_guard<std::mutex> lk(hc::g_words_mu);
        readers = hc::error_readers();
    }
    for (auto reader : readers) {
        const char* name = "";
        uint32_t word = reader(&name);
        if (word != 0)
            return fail(HC_ERR_TIMEOUT, "%s: bounded wait expired (error word 0x%08x)", name, word);
    }
    return ok();
}

const char* hc_last_error_string(void) { return hc::t_last_msg; }

int hc_last_error(void) { return hc::t_last_status; }

int hc_set_fault(const char* spec) {
    std::lock_guard<std::mutex> lk(hc::g_fault_mu);
    hc::g_fault_env_read = true;
    hc::parse_fault(spec);
    return ok();
}

}  // extern "C"
