// C++ device runtime of the harness on B200, built on the C-ABI in hc_runtime.h.
//
// Mirrors the reference's device layer so that its host code (runners, tests, benches) keeps
// compiling with the same calls:
//   include/harness/ascend_runtime.hpp:16-92  RuntimeInit ... EventSynchronize, DeviceMemory RAII
//   include/harness/skip.hpp:20-27            IsAscendRuntimeAvailable / HasUsableDevice /
//                                             GetDeviceCount
// Same names, arguments and error behaviour: free functions report failure through their return
// value (false / nullptr / 0) and never throw; DeviceMemory(size) throws std::runtime_error when
// the allocation fails.  `harness::ascend` is an alias of `harness::device`, so code written
// against the reference header compiles unchanged.
//
// Differences, all deliberate:
//   * the device is a CUDA GPU; SetDevice / GetCurrentDevice act on the calling thread (CUDA
//     semantics), so one host thread per GPU can drive several GPUs; the reference kept one
//     global device (src/ascend_runtime.cpp:170-172);
//   * events are real CUDA events (the reference stubbed them, src/ascend_runtime.cpp:238-243);
//   * MemcpyHostToDevice / MemcpyDeviceToHost stay synchronous like the reference's; the
//     *Async variants take a stream;
//   * GetErrorString maps an hc_status code to its name and LastErrorMessage() gives the
//     detailed message of the calling thread's last failure.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>

namespace harness {
namespace device {

// ---- runtime and devices (ascend_runtime.hpp:16-22) ----
bool RuntimeInit();
bool RuntimeFinalize();
int GetDeviceCount();
bool SetDevice(int device_id);
int GetCurrentDevice();

// ---- streams (ascend_runtime.hpp:25-30) ----
struct StreamDeleter {
    void operator()(void* stream) const;
};
using StreamHandle = std::unique_ptr<void, StreamDeleter>;
StreamHandle CreateStream();
bool StreamSynchronize(void* stream);
bool DeviceSynchronize();

// ---- memory (ascend_runtime.hpp:33-38) ----
void* DeviceMalloc(size_t size);
void DeviceFree(void* ptr);
bool MemcpyHostToDevice(void* dst, const void* src, size_t size);
bool MemcpyDeviceToHost(void* dst, const void* src, size_t size);
bool MemcpyHostToDeviceAsync(void* dst, const void* src, size_t size, void* stream);
bool MemcpyDeviceToHostAsync(void* dst, const void* src, size_t size, void* stream);
// Page-locked host memory (copies from it overlap kernels); nullptr on failure.
void* HostMallocPinned(size_t size);
void HostFreePinned(void* ptr);

// ---- errors (ascend_runtime.hpp:41-42) ----
const char* GetErrorString(int error_code);
int GetLastError();
std::string LastErrorMessage();
// Reads and clears the device error words of bounded spin-waits; false when a kernel on the
// current device gave up a wait since the last check (then GetLastError() == HC_ERR_TIMEOUT).
bool CheckDeviceError();

// ---- environment (ascend_runtime.hpp:45-47) ----
bool IsAvailable();
std::string GetDriverVersion();
std::string GetSocVersion();  // device name and compute capability, e.g. "NVIDIA B200 (sm_100)"

// ---- device memory RAII (ascend_runtime.hpp:52-80) ----
class DeviceMemory {
public:
    DeviceMemory() = default;
    explicit DeviceMemory(size_t size) : ptr_(DeviceMalloc(size)), size_(size) {
        if (!ptr_ && size > 0) throw std::runtime_error("DeviceMalloc failed: " + LastErrorMessage());
    }
    ~DeviceMemory() { reset(); }

    DeviceMemory(const DeviceMemory&) = delete;
    DeviceMemory& operator=(const DeviceMemory&) = delete;
    DeviceMemory(DeviceMemory&& other) noexcept : ptr_(other.ptr_), size_(other.size_) {
        other.ptr_ = nullptr;
        other.size_ = 0;
    }
    DeviceMemory& operator=(DeviceMemory&& other) noexcept {
        if (this != &other) {
            reset();
            ptr_ = other.ptr_;
            size_ = other.size_;
            other.ptr_ = nullptr;
            other.size_ = 0;
        }
        return *this;
    }

    void* data() { return ptr_; }
    const void* data() const { return ptr_; }
    size_t size() const { return size_; }
    explicit operator bool() const { return ptr_ != nullptr; }
    template <typename T>
    T* as() { return static_cast<T*>(ptr_); }

private:
    void reset() {
        if (ptr_) DeviceFree(ptr_);
        ptr_ = nullptr;
        size_ = 0;
    }
    void* ptr_ = nullptr;
    size_t size_ = 0;
};

// ---- events (ascend_runtime.hpp:85-92) ----
struct EventDeleter {
    void operator()(void* event) const;
};
using EventHandle = std::unique_ptr<void, EventDeleter>;
EventHandle CreateEvent();
bool RecordEvent(void* event, void* stream);
bool EventElapsedTime(float* ms, void* start_event, void* end_event);
bool EventSynchronize(void* event);

}  // namespace device

// The reference's runners and tests name the device layer harness::ascend.
namespace ascend = device;

// ---- skip helpers (include/harness/skip.hpp:20-27) ----
bool IsDeviceRuntimeAvailable();
bool HasUsableDevice();
int GetDeviceCount();
inline bool IsAscendRuntimeAvailable() { return IsDeviceRuntimeAvailable(); }

}  // namespace harness
