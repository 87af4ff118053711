/*
 * hc_runtime.h -- C-ABI device runtime shim for the B200 operator ladder.
 *
 * Replaces the harness's Ascend device layer:
 *   include/harness/ascend_runtime.hpp:16-92  (RuntimeInit, GetDeviceCount, SetDevice,
 *       CreateStream, StreamSynchronize, DeviceMalloc/Free, MemcpyH2D/D2H, CreateEvent,
 *       RecordEvent, EventElapsedTime, EventSynchronize)
 *   src/ascend_runtime.cpp:1-264              (dlopen'd libascendcl implementation)
 *   include/harness/skip.hpp:20-27            (IsAscendRuntimeAvailable / HasUsableDevice)
 *
 * Conventions
 *   - Every entry point returns an int status: 0 (HC_OK) on success, a positive hc_status
 *     otherwise.  hc_last_error_string() describes the most recent failure of the calling
 *     thread.  Nothing throws across this boundary.
 *   - Pointers are plain addresses.  Device pointers may come from hc_malloc or from any other
 *     allocator of the same CUDA context (e.g. a framework's caching allocator).
 *   - "stream" is a cudaStream_t passed as void*; NULL means the legacy default stream and
 *     makes the memcpy helpers synchronous, like the reference's blocking aclrtMemcpy.
 *   - hc_set_device() is per calling thread (CUDA semantics).  The reference kept one global
 *     device (src/ascend_runtime.cpp:170-172); one host thread per GPU is the intended use.
 *   - The caller owns every buffer.  The shim allocates nothing behind the caller's back.
 *
 * Host-side fault injection (for failure-path tests, no GPU fault involved):
 *   environment HC_FAULT="<call>:<n>" makes the n-th (1-based) call of <call> return
 *   HC_ERR_INJECTED without touching the device.  <call> is one of malloc, memcpy, launch.
 */
#ifndef HC_RUNTIME_H
#define HC_RUNTIME_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum hc_status {
    HC_OK = 0,
    HC_ERR_INVALID = 1,      /* bad argument: null pointer, zero/unsupported size, bad enum */
    HC_ERR_CUDA = 2,         /* a CUDA runtime/driver call failed; see hc_last_error_string() */
    HC_ERR_UNSUPPORTED = 3,  /* shape/dtype combination this library has no kernel for */
    HC_ERR_TIMEOUT = 4,      /* a kernel's bounded wait expired (device error word was set) */
    HC_ERR_NO_DEVICE = 5,    /* no CUDA device visible */
    HC_ERR_INJECTED = 6      /* failure injected through HC_FAULT */
} hc_status;

/* Element types; numbering follows harness::Dtype (include/harness/dtype.hpp:9-16). */
typedef enum hc_dtype {
    HC_DTYPE_F32 = 0,
    HC_DTYPE_F16 = 1,
    HC_DTYPE_BF16 = 2,
    HC_DTYPE_I32 = 3,
    HC_DTYPE_I8 = 4,
    HC_DTYPE_U8 = 5
} hc_dtype;

/* ascend::RuntimeInit / IsAvailable (ascend_runtime.hpp:16,45). */
int hc_init(void);
/* ascend::GetDeviceCount (ascend_runtime.hpp:20). Writes 0 and returns HC_ERR_NO_DEVICE when none. */
int hc_device_count(int* count);
/* ascend::SetDevice / GetCurrentDevice (ascend_runtime.hpp:21-22). */
int hc_set_device(int device);
int hc_get_device(int* device);
/* ascend::GetDriverVersion (ascend_runtime.hpp:46): CUDA driver version, e.g. 12090. */
int hc_driver_version(int* version);
/* Streaming-multiprocessor count and name of the current device. */
int hc_device_sm_count(int* sms);
int hc_device_name(char* buf, size_t buflen);

/* ascend::DeviceMalloc / DeviceFree (ascend_runtime.hpp:33-34). */
int hc_malloc(void** ptr, size_t bytes);
int hc_free(void* ptr);
/* Page-locked host buffers for overlapped host<->device copies (no reference counterpart). */
int hc_malloc_host(void** ptr, size_t bytes);
int hc_free_host(void* ptr);

/* ascend::MemcpyHostToDevice / MemcpyDeviceToHost (ascend_runtime.hpp:37-38), plus d2d. */
int hc_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int hc_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int hc_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
int hc_memset(void* dst, int value, size_t bytes, void* stream);

/* ascend::CreateStream / StreamSynchronize / StreamDeleter (ascend_runtime.hpp:25-30). */
int hc_stream_create(void** stream);
int hc_stream_destroy(void* stream);
int hc_stream_sync(void* stream);
int hc_device_sync(void);

/* ascend::CreateEvent / RecordEvent / EventElapsedTime / EventSynchronize
 * (ascend_runtime.hpp:85-92).  The reference stubbed these (src/ascend_runtime.cpp:238-243);
 * here they are real CUDA events. */
int hc_event_create(void** event);
int hc_event_destroy(void* event);
int hc_event_record(void* event, void* stream);
int hc_event_sync(void* event);
int hc_event_elapsed_ms(float* ms, void* start_event, void* end_event);

/* Reads and clears the device-side error words that bounded spin-waits set when they expire.
 * Returns HC_OK when no kernel on the current device reported a timeout since the last call,
 * HC_ERR_TIMEOUT otherwise (hc_last_error_string() then names the kernel and wait site). */
int hc_check_device_error(void);

/* Diagnostic: launches one CTA whose mbarrier wait can never complete, with the same bounded-wait
 * code the tensor-core kernels use and a budget of `budget_us` microseconds (1..1e6).  The wait
 * gives up, the kernel exits normally and the call returns HC_ERR_TIMEOUT (error word read and
 * cleared).  Proves on a real device that an expired wait is reported, not hung on. */
int hc_selftest_bounded_wait(uint32_t budget_us);

/* ascend::GetErrorString / GetLastError (ascend_runtime.hpp:41-42), thread-local. */
const char* hc_last_error_string(void);
int hc_last_error(void);

/* Fault injection control for tests: same syntax as the HC_FAULT environment variable;
 * NULL or "" disarms.  Counts restart at every call. */
int hc_set_fault(const char* spec);

#ifdef __cplusplus
}
#endif

#endif /* HC_RUNTIME_H */
