// Host-side plumbing shared by the C ABI's source files: the device and encoder objects, typed errors raised as
// exceptions inside the library and turned into og_status at the boundary (guard), and the argument checks every
// kernel family uses (KernelSupport.cs:75-130 Check.Range / RangeBytes / Product, IndexSupport.cs:47-55 Axis).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/onegpu_cuda.h"

struct og_device {
    int ordinal = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = true;
    int sm_count = 0;
    cudaDeviceProp prop = {};
    int* status = nullptr;       // device word a kernel sets when a bounded wait gave up
    int* status_host = nullptr;  // pinned mirror for readbacks
    cudaStream_t upload = nullptr;    // copy-engine stream of og_buffer_write_async
    cudaStream_t readback = nullptr;  // copy-engine stream of og_buffer_read_async
    // Pinned status words of the asynchronous readbacks (one per readback in flight), page-locked once with the
    // device: locking a word per readback and releasing it at the wait (cudaFreeHost synchronises the whole device)
    // would drain the transfer pipeline at every wait, so the uploads of the next step could not overlap the readback
    // of the last one.
    int* readback_words = nullptr;
    std::vector<int> readback_free;  // indices of the unused words
    std::mutex readback_mu;
};

constexpr int kReadbackWords = 1024;

// One recorded piece of work: launches on the stream it is given.
using OgOp = std::function<cudaError_t(cudaStream_t)>;

struct og_encoder {
    og_device* device = nullptr;
    std::vector<OgOp> ops;
    int64_t dispatches = 0;
};

namespace og_host {

struct OgError {
    og_status status;
    std::string operation, argument, message, capability, expected, actual;
};

constexpr int64_t kMaxElements = 2147483647;  // Check.MaxElements: sizes stay below int.MaxValue

void set_last(const OgError& e);
[[noreturn]] void shape(const char* op, const std::string& arg, const std::string& msg);
[[noreturn]] void null_arg(const char* op, const std::string& arg);
[[noreturn]] void unsupported(const char* op, const std::string& msg, const std::string& cap, const std::string& exp,
                              const std::string& act);
// cudaErrorMemoryAllocation -> OG_ERROR_OUT_OF_MEMORY, sticky errors -> OG_ERROR_DEVICE_LOST, others OG_ERROR_CUDA.
void check_cuda(cudaError_t e, const char* what);
void use(og_device* d);
const char* type_name(int32_t t);
int elem_size(int32_t t);

// Check.Range: offset not negative, [offset, offset + extent) inside the buffer (errors name+"Offset" / name).
void range(const char* op, const std::string& name, int64_t length, int32_t offset, int64_t extent);

// Check.Range with half = true: additionally the 32-bit word holding the last half lies inside the buffer.
inline void range_half(const char* op, const std::string& name, int64_t length, int32_t offset, int64_t extent) {
    range(op, name, length, offset, extent);
    if (extent > 0 && (((static_cast<int64_t>(offset) + extent + 1) >> 1) << 1) > length)
        shape(op, name, "the buffer of " + std::to_string(length) +
                            " halves ends inside a 32-bit word; allocate GpuKernelBuffers.PaddedHalfLength(n) elements");
}

// Check.RangeBytes: additionally the 32-bit word holding the last byte lies inside the buffer.
inline void range_bytes(const char* op, const std::string& name, int64_t length, int32_t offset, int64_t extent) {
    range(op, name, length, offset, extent);
    if (extent > 0 && (((static_cast<int64_t>(offset) + extent + 3) >> 2) << 2) > length)
        shape(op, name, "the buffer of " + std::to_string(length) +
                            " bytes ends inside a 32-bit word; allocate GpuKernelBuffers.PaddedBoolLength(n) elements");
}

// Check.Product: the element count of a shape; every dimension non-negative, the product at most kMaxElements.
inline int64_t product(const char* op, const std::string& name, const int32_t* dims, int32_t rank) {
    int64_t n = 1;
    for (int32_t i = 0; i < rank; i++) {
        const std::string arg = name + "[" + std::to_string(i) + "]";
        if (dims[i] < 0) shape(op, arg, "dimension " + std::to_string(dims[i]) + " is negative");
        n *= dims[i];
        if (n > kMaxElements)
            shape(op, arg, "the tensor holds more than " + std::to_string(kMaxElements) + " elements");
    }
    return n;
}

// IndexSupport.Axis: an axis in [-rank, rank), returned non-negative.
inline int32_t axis_of(const char* op, int32_t axis, int32_t rank) {
    if (axis < -rank || axis >= rank)
        shape(op, "axis",
              "axis " + std::to_string(axis) + " is outside [" + std::to_string(-rank) + ", " + std::to_string(rank) + ")");
    return axis < 0 ? axis + rank : axis;
}

template <class F>
og_status guard(F&& f) {
    try {
        f();
        return OG_OK;
    } catch (const OgError& e) {
        set_last(e);
        return e.status;
    } catch (const std::bad_alloc&) {
        set_last(OgError{OG_ERROR_OUT_OF_MEMORY, "host", "", "host allocation failed", "", "", ""});
        return OG_ERROR_OUT_OF_MEMORY;
    } catch (...) {
        set_last(OgError{OG_ERROR_CUDA, "host", "", "unexpected failure", "", "", ""});
        return OG_ERROR_CUDA;
    }
}

}  // namespace og_host
