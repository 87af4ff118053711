// harness::device runtime on top of the C-ABI (hc_runtime.h).  Every function maps one-to-one
// onto a C entry point and turns its status into the reference's bool / pointer / int return
// conventions (include/harness/ascend_runtime.hpp:16-92, src/ascend_runtime.cpp:165-262).
#include "harness/device_runtime.hpp"

#include "hc_runtime.h"

namespace harness {
namespace device {

bool RuntimeInit() { return hc_init() == HC_OK; }

// CUDA's primary context lives until the process exits; there is nothing to tear down per call.
bool RuntimeFinalize() { return true; }

int GetDeviceCount() {
    int n = 0;
    return hc_device_count(&n) == HC_OK ? n : 0;
}

bool SetDevice(int device_id) { return hc_set_device(device_id) == HC_OK; }

int GetCurrentDevice() {
    int d = -1;
    return hc_get_device(&d) == HC_OK ? d : -1;
}

void StreamDeleter::operator()(void* stream) const {
    if (stream) hc_stream_destroy(stream);
}

StreamHandle CreateStream() {
    void* s = nullptr;
    if (hc_stream_create(&s) != HC_OK) return StreamHandle(nullptr);
    return StreamHandle(s);
}

bool StreamSynchronize(void* stream) { return hc_stream_sync(stream) == HC_OK; }

bool DeviceSynchronize() { return hc_device_sync() == HC_OK; }

void* DeviceMalloc(size_t size) {
    if (size == 0) return nullptr;
    void* p = nullptr;
    return hc_malloc(&p, size) == HC_OK ? p : nullptr;
}

void DeviceFree(void* ptr) {
    if (ptr) hc_free(ptr);
}

bool MemcpyHostToDevice(void* dst, const void* src, size_t size) {
    return size == 0 || hc_memcpy_h2d(dst, src, size, nullptr) == HC_OK;
}

bool MemcpyDeviceToHost(void* dst, const void* src, size_t size) {
    return size == 0 || hc_memcpy_d2h(dst, src, size, nullptr) == HC_OK;
}

bool MemcpyHostToDeviceAsync(void* dst, const void* src, size_t size, void* stream) {
    return size == 0 || hc_memcpy_h2d(dst, src, size, stream) == HC_OK;
}

bool MemcpyDeviceToHostAsync(void* dst, const void* src, size_t size, void* stream) {
    return size == 0 || hc_memcpy_d2h(dst, src, size, stream) == HC_OK;
}

void* HostMallocPinned(size_t size) {
    if (size == 0) return nullptr;
    void* p = nullptr;
    return hc_malloc_host(&p, size) == HC_OK ? p : nullptr;
}

void HostFreePinned(void* ptr) {
    if (ptr) hc_free_host(ptr);
}

const char* GetErrorString(int error_code) {
    switch (error_code) {
        case HC_OK: return "HC_OK";
        case HC_ERR_INVALID: return "HC_ERR_INVALID";
        case HC_ERR_CUDA: return "HC_ERR_CUDA";
        case HC_ERR_UNSUPPORTED: return "HC_ERR_UNSUPPORTED";
        case HC_ERR_TIMEOUT: return "HC_ERR_TIMEOUT";
        case HC_ERR_NO_DEVICE: return "HC_ERR_NO_DEVICE";
        case HC_ERR_INJECTED: return "HC_ERR_INJECTED";
        default: return "unknown hc_status";
    }
}

int GetLastError() { return hc_last_error(); }

std::string LastErrorMessage() {
    const char* m = hc_last_error_string();
    return m ? std::string(m) : std::string();
}

bool CheckDeviceError() { return hc_check_device_error() == HC_OK; }

bool IsAvailable() { return GetDeviceCount() > 0; }

std::string GetDriverVersion() {
    int v = 0;
    if (hc_driver_version(&v) != HC_OK) return std::string();
    return std::to_string(v / 1000) + "." + std::to_string((v % 1000) / 10);
}

std::string GetSocVersion() {
    char buf[256];
    if (hc_device_name(buf, sizeof(buf)) != HC_OK) return std::string();
    return std::string(buf);
}

void EventDeleter::operator()(void* event) const {
    if (event) hc_event_destroy(event);
}

EventHandle CreateEvent() {
    void* e = nullptr;
    if (hc_event_create(&e) != HC_OK) return EventHandle(nullptr);
    return EventHandle(e);
}

bool RecordEvent(void* event, void* stream) { return hc_event_record(event, stream) == HC_OK; }

bool EventElapsedTime(float* ms, void* start_event, void* end_event) {
    return hc_event_elapsed_ms(ms, start_event, end_event) == HC_OK;
}

bool EventSynchronize(void* event) { return hc_event_sync(event) == HC_OK; }

}  // namespace device

bool IsDeviceRuntimeAvailable() { return device::GetDeviceCount() > 0; }

bool HasUsableDevice() { return device::GetDeviceCount() > 0 && device::RuntimeInit(); }

int GetDeviceCount() { return device::GetDeviceCount(); }

}  // namespace harness
