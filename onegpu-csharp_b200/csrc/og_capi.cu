// Host layer and C ABI of libonegpu_cuda.so: the compute subset of GpuDevice on CUDA (devices, buffers, uploads and
// readbacks, encoders replayed on a stream, timestamps from CUDA events), the argument checks of Int8Gemm and
// DynamicQuantizeKernels in the reference's order with its argument names, and the dispatch to the kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/onegpu_cuda.h"
#include "og_gemm.h"
#include "og_host.h"
#include "og_ptx.cuh"

// ---- errors ---------------------------------------------------------------------------------------------------------

namespace og_host {

thread_local og_error_info g_last = {};

void copy_field(char* dst, size_t cap, const std::string& s) {
    const size_t n = std::min(cap - 1, s.size());
    memcpy(dst, s.data(), n);
    dst[n] = 0;
}

void set_last(const OgError& e) {
    og_error_info info = {};
    info.status = e.status;
    copy_field(info.operation, sizeof(info.operation), e.operation);
    copy_field(info.argument, sizeof(info.argument), e.argument);
    copy_field(info.message, sizeof(info.message), e.message);
    copy_field(info.capability, sizeof(info.capability), e.capability);
    copy_field(info.expected, sizeof(info.expected), e.expected);
    copy_field(info.actual, sizeof(info.actual), e.actual);
    g_last = info;
}

[[noreturn]] void shape(const char* op, const std::string& arg, const std::string& msg) {
    throw OgError{OG_ERROR_SHAPE, op, arg, msg, "", "", ""};
}

[[noreturn]] void null_arg(const char* op, const std::string& arg) {
    throw OgError{OG_ERROR_ARGUMENT_NULL, op, arg, "Value cannot be null.", "", "", ""};
}

[[noreturn]] void unsupported(const char* op, const std::string& msg, const std::string& cap, const std::string& exp,
                              const std::string& act) {
    throw OgError{OG_ERROR_UNSUPPORTED, op, "", msg, cap, exp, act};
}

bool sticky(cudaError_t e) {
    switch (e) {
        case cudaErrorIllegalAddress:
        case cudaErrorLaunchFailure:
        case cudaErrorHardwareStackError:
        case cudaErrorIllegalInstruction:
        case cudaErrorMisalignedAddress:
        case cudaErrorInvalidAddressSpace:
        case cudaErrorInvalidPc:
        case cudaErrorECCUncorrectable:
        case cudaErrorAssert:
        case cudaErrorLaunchTimeout:
        case cudaErrorUnknown:
            return true;
        default:
            return false;
    }
}

void check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    og_status st = e == cudaErrorMemoryAllocation ? OG_ERROR_OUT_OF_MEMORY
                   : sticky(e)                     ? OG_ERROR_DEVICE_LOST
                                                   : OG_ERROR_CUDA;
    throw OgError{st, what, "", std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e), "", "", ""};
}


void put_string(char* buf, uint64_t cap, const std::string& s) {
    if (buf == nullptr || cap == 0) return;
    copy_field(buf, static_cast<size_t>(cap), s);
}

void use(og_device* d) { check_cuda(cudaSetDevice(d->ordinal), "cudaSetDevice"); }

const char* type_name(int32_t t) {
    switch (t) {
        case OG_U8: return "Byte";
        case OG_S8: return "SByte";
        case OG_I32: return "Int32";
        case OG_F32: return "Single";
        case OG_F16: return "Half";
        case OG_U32: return "UInt32";
        case OG_U16: return "UInt16";
        case OG_I16: return "Int16";
        case OG_I64: return "Int64";
        default: return "Unknown";
    }
}

int elem_size(int32_t t) {
    switch (t) {
        case OG_U8:
        case OG_S8: return 1;
        case OG_F16:
        case OG_U16:
        case OG_I16: return 2;
        case OG_I64: return 8;
        default: return 4;
    }
}

// Check.Range: offset not negative, [offset, offset + extent) inside the buffer.
void range(const char* op, const std::string& name, int64_t length, int32_t offset, int64_t extent) {
    if (offset < 0) shape(op, name + "Offset", "offset " + std::to_string(offset) + " is negative");
    if (extent < 0 || static_cast<int64_t>(offset) + extent > length)
        shape(op, name,
              "elements " + std::to_string(offset) + ".." + std::to_string(static_cast<int64_t>(offset) + extent) +
                  " reach past the buffer of " + std::to_string(length));
}

}  // namespace og_host

using namespace og_host;

// ---- objects ----------------------------------------------------------------------------------------------------

using Op = OgOp;

struct og_readback {
    og_device* device = nullptr;
    cudaEvent_t done = nullptr;
    int* status_host = nullptr;  // the device's failure word as it stood when the copy ran
    int word = -1;               // its index among the device's pinned words, or -1 when it was page-locked alone
};

namespace {

// A pinned word for one readback: one of the device's, or (all of them in flight) one of its own.
void take_status_word(og_device* d, og_readback* r) {
    {
        std::lock_guard<std::mutex> g(d->readback_mu);
        if (!d->readback_free.empty()) {
            r->word = d->readback_free.back();
            d->readback_free.pop_back();
            r->status_host = d->readback_words + r->word;
            return;
        }
    }
    check_cuda(cudaMallocHost(&r->status_host, sizeof(int)), "ReadAsync");
}

void give_status_word(og_readback* r) {
    if (r->word >= 0) {
        std::lock_guard<std::mutex> g(r->device->readback_mu);
        r->device->readback_free.push_back(r->word);
    } else if (r->status_host != nullptr) {
        cudaFreeHost(r->status_host);
    }
    r->status_host = nullptr;
}

}  // namespace

struct og_graph {
    og_device* device = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

struct og_timestamps {
    og_device* device = nullptr;
    std::vector<cudaEvent_t> events;
};

struct og_int8_gemm {
    og_device* device = nullptr;
    bool allow_dot = true;
    int kernel = OG_KERNEL_AUTO;
    int tile = 0;
    int stream_k = 0;  // 0: whole tiles + the split tail of int32 products; 1: whole tiles only; 2: stream-K
    std::string variant;
    std::string last = "none";
    std::vector<void*> scratch;  // int32 byte-sum buffers; older ones live until destroy (recorded work may name them)
    int64_t scratch_elements = 0;
    void* sk_buf = nullptr;      // stream-K hand-over buffer of the tensor-core product, allocated on first need
    int64_t sk_bytes = 0;
    // Pitched copies of operands that TMA cannot load in place (A, B; the latest of each; older ones live until destroy)
    void* stage[2] = {nullptr, nullptr};
    int64_t stage_bytes[2] = {0, 0};
    // Partials and tickets of the evenly split few-rows product (the latest pair; older ones live until destroy)
    std::vector<void*> rows_bufs;
    int32_t* rows_part = nullptr;
    unsigned int* rows_ticket = nullptr;
    int64_t rows_part_ints = 0, rows_ticket_count = 0;
};

struct og_dynamic_quantize {
    og_device* device = nullptr;
    og::DqScratch* scratch = nullptr;
};

namespace {

// Reads the kernels' failure word of the device (after the stream has drained) and clears it.
void check_device_status(og_device* d) {
    check_cuda(cudaMemcpyAsync(d->status_host, d->status, sizeof(int), cudaMemcpyDeviceToHost, d->stream),
               "status readback");
    check_cuda(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
    if (*d->status_host != 0) {
        check_cuda(cudaMemsetAsync(d->status, 0, sizeof(int), d->stream), "status reset");
        check_cuda(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
        throw OgError{OG_ERROR_COMMAND_FAILED, "GpuDevice", "",
                      "a kernel gave up waiting on its own pipeline (watchdog) and skipped its work", "Watchdog", "",
                      ""};
    }
}

// ---- argument checks (Int8Gemm.cs:393-501, KernelSupport.cs:75-91) -------------------------------------------------

const char* kGemm = "Int8Gemm";
const char* kDq = "DynamicQuantizeLinear";



void require_int8(const og_buffer* b, const char* arg) {
    if (b->type != OG_U8 && b->type != OG_S8)
        shape(kGemm, arg,
              std::string("element type ") + type_name(b->type) +
                  " is not supported; use byte (uint8) or sbyte (int8)");
}

void require_type(const char* op, const og_buffer* b, const char* arg, int32_t want) {
    if (b->type != want)
        shape(op, arg, std::string("element type ") + type_name(b->type) + " is not supported; use " +
                           type_name(want));
}

void non_negative(const char* arg, int32_t v) {
    if (v < 0) shape(kGemm, arg, "must not be negative, got " + std::to_string(v));
}

// CheckVector: the buffer exists and holds one value, or n from the offset.
void check_vector(const char* name, const og_operand* o, int32_t n) {
    if (o->buffer.ptr == nullptr) null_arg(kGemm, name);
    range(kGemm, name, o->buffer.length, o->offset, o->is_vector ? n : 1);
}

// CheckVector with isVector = true: biases are always one value per column (Int8Gemm.cs:242,296,656), whatever the
// operand's IsVector says; the kernels read bias[n] for every column n.
void check_column_vector(const char* name, const og_operand* o, int32_t n) {
    if (o->buffer.ptr == nullptr) null_arg(kGemm, name);
    range(kGemm, name, o->buffer.length, o->offset, n);
}

// CheckRange of an operand matrix.
void check_matrix(const char* operand, int32_t offset, int32_t stride, int32_t rows, int32_t cols, int64_t ld,
                  int32_t batch, int64_t length) {
    const int64_t last = offset + static_cast<int64_t>(batch - 1) * stride + static_cast<int64_t>(rows - 1) * ld +
                         (cols - 1);
    if (last >= length)
        shape(kGemm, std::string("Offset") + operand,
              std::string("operand ") + operand + " reaches byte " + std::to_string(last) + " but its buffer holds " +
                  std::to_string(length));
}

struct Prepared {
    int64_t lda, ldb;
    bool ok;
};

// Prepare (Int8Gemm.cs:419-484) without the encoder check.
Prepared prepare(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b, const og_operand* za,
                 const og_operand* zb) {
    if (a == nullptr || a->ptr == nullptr) null_arg(kGemm, "a");
    if (b == nullptr || b->ptr == nullptr) null_arg(kGemm, "b");
    if (p == nullptr) null_arg(kGemm, "problem");
    require_int8(a, "a");
    require_int8(b, "b");
    non_negative("M", p->m);
    non_negative("N", p->n);
    non_negative("K", p->k);
    non_negative("OffsetA", p->offset_a);
    non_negative("OffsetB", p->offset_b);
    non_negative("OffsetC", p->offset_c);
    non_negative("StrideA", p->stride_a);
    non_negative("StrideB", p->stride_b);
    non_negative("Lda", p->lda);
    non_negative("Ldb", p->ldb);
    if (p->batch < 1) shape(kGemm, "Batch", "must be at least 1, got " + std::to_string(p->batch));
    const int64_t lda = p->lda == 0 ? std::max(p->k, 1) : p->lda;
    const int64_t cols_b = p->transpose_b ? p->k : p->n;
    const int64_t rows_b = p->transpose_b ? p->n : p->k;
    const int64_t ldb = p->ldb == 0 ? std::max<int64_t>(cols_b, 1) : p->ldb;
    if (lda < p->k) shape(kGemm, "Lda", std::to_string(lda) + " is smaller than K = " + std::to_string(p->k));
    if (ldb < cols_b)
        shape(kGemm, "Ldb", std::to_string(ldb) + " is smaller than the stored row length " + std::to_string(cols_b));
    const __int128 elems = static_cast<__int128>(p->batch) * p->m * p->n;
    if (elems > kMaxElements) shape(kGemm, "Batch", "the result holds more elements than the kernels address");
    if (p->m > 0 && p->n > 0 && p->k > 0) {
        check_matrix("A", p->offset_a, p->stride_a, p->m, p->k, lda, p->batch, a->length);
        check_matrix("B", p->offset_b, p->stride_b, static_cast<int32_t>(rows_b), static_cast<int32_t>(cols_b), ldb,
                     p->batch, b->length);
    }
    if (za != nullptr) {
        check_vector("zpA", za, p->m);
        if (za->buffer.type != a->type) require_type(kGemm, &za->buffer, "zpA", a->type);
    }
    if (zb != nullptr) {
        check_vector("zpB", zb, p->n);
        if (zb->buffer.type != b->type) require_type(kGemm, &zb->buffer, "zpB", b->type);
    }
    return Prepared{lda, ldb, p->m > 0 && p->n > 0};
}

int64_t result_count(const og_int8_gemm_problem* p) { return static_cast<int64_t>(p->batch) * p->m * p->n; }

Prepared check_int32(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b, const og_buffer* c,
                     const og_operand* za, const og_operand* zb, const og_operand* bias) {
    if (c == nullptr || c->ptr == nullptr) null_arg(kGemm, "c");
    Prepared pr = prepare(p, a, b, za, zb);
    require_type(kGemm, c, "c", OG_I32);
    range(kGemm, "c", c->length, p->offset_c, result_count(p));
    if (bias != nullptr) {
        check_column_vector("bias", bias, p->n);
        require_type(kGemm, &bias->buffer, "bias", OG_I32);
    }
    return pr;
}

Prepared check_float(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b, const og_buffer* c,
                     const og_operand* scale, const og_operand* za, const og_operand* zb, const og_operand* fbias,
                     const og_operand* ibias) {
    if (c == nullptr || c->ptr == nullptr) null_arg(kGemm, "c");
    Prepared pr = prepare(p, a, b, za, zb);
    require_type(kGemm, c, "c", OG_F32);
    range(kGemm, "c", c->length, p->offset_c, result_count(p));
    if (scale == nullptr) null_arg(kGemm, "scale");
    check_vector("scale", scale, p->n);
    require_type(kGemm, &scale->buffer, "scale", OG_F32);
    if (fbias != nullptr) {
        check_column_vector("floatBias", fbias, p->n);
        require_type(kGemm, &fbias->buffer, "floatBias", OG_F32);
    }
    if (!pr.ok) return pr;
    if (ibias != nullptr) {
        check_column_vector("intBias", ibias, p->n);
        require_type(kGemm, &ibias->buffer, "intBias", OG_I32);
    }
    return pr;
}

// The float form with the scale formed as scaleA * scaleB[n]: EncodeFloat's checks with "bScale" for the scale,
// plus one value of "aScale".
Prepared check_dequantize(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b, const og_buffer* c,
                          const og_operand* a_scale, const og_operand* b_scale, const og_operand* za,
                          const og_operand* zb, const og_operand* fbias, const og_operand* ibias) {
    if (c == nullptr || c->ptr == nullptr) null_arg(kGemm, "c");
    Prepared pr = prepare(p, a, b, za, zb);
    require_type(kGemm, c, "c", OG_F32);
    range(kGemm, "c", c->length, p->offset_c, result_count(p));
    if (a_scale == nullptr) null_arg(kGemm, "aScale");
    if (b_scale == nullptr) null_arg(kGemm, "bScale");
    if (a_scale->is_vector) shape(kGemm, "aScale", "must be one value (the scale of the whole of A)");
    check_vector("aScale", a_scale, p->n);
    require_type(kGemm, &a_scale->buffer, "aScale", OG_F32);
    check_vector("bScale", b_scale, p->n);
    require_type(kGemm, &b_scale->buffer, "bScale", OG_F32);
    if (fbias != nullptr) {
        check_column_vector("floatBias", fbias, p->n);
        require_type(kGemm, &fbias->buffer, "floatBias", OG_F32);
    }
    if (!pr.ok) return pr;
    if (ibias != nullptr) {
        check_column_vector("intBias", ibias, p->n);
        require_type(kGemm, &ibias->buffer, "intBias", OG_I32);
    }
    return pr;
}

Prepared check_requantized(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b, const og_buffer* y,
                           const og_operand* mult, int32_t zero_y, const og_operand* za, const og_operand* zb,
                           const og_operand* ibias, const og_operand* scratch) {
    if (y == nullptr || y->ptr == nullptr) null_arg(kGemm, "y");
    Prepared pr = prepare(p, a, b, za, zb);
    require_int8(y, "y");
    const bool out_signed = y->type == OG_S8;
    if (zero_y < (out_signed ? -128 : 0) || zero_y > (out_signed ? 127 : 255))
        shape(kGemm, "zeroPointY", std::to_string(zero_y) + " is outside the output type's range");
    const int64_t count = result_count(p);
    range(kGemm, "y", y->length, p->offset_c, count);
    if (mult == nullptr) null_arg(kGemm, "multiplier");
    check_vector("multiplier", mult, p->n);
    require_type(kGemm, &mult->buffer, "multiplier", OG_F32);
    if (!pr.ok) return pr;
    if (scratch != nullptr) {
        if (scratch->buffer.ptr == nullptr) null_arg(kGemm, "given");
        range(kGemm, "scratch", scratch->buffer.length, scratch->offset, count);
        require_type(kGemm, &scratch->buffer, "scratch", OG_I32);
    }
    if (ibias != nullptr) {
        check_column_vector("intBias", ibias, p->n);
        require_type(kGemm, &ibias->buffer, "intBias", OG_I32);
    }
    return pr;
}

void check_dq(const og_buffer* x, int32_t offset_x, int32_t count, const og_buffer* y, int32_t offset_y,
              const og_buffer* scale, int32_t offset_scale, const og_buffer* zp, int32_t offset_zp) {
    if (x == nullptr || x->ptr == nullptr) null_arg(kDq, "x");
    if (y == nullptr || y->ptr == nullptr) null_arg(kDq, "y");
    if (scale == nullptr || scale->ptr == nullptr) null_arg(kDq, "scale");
    if (zp == nullptr || zp->ptr == nullptr) null_arg(kDq, "zeroPoint");
    require_type(kDq, x, "x", OG_F32);
    require_type(kDq, y, "y", OG_U8);
    require_type(kDq, scale, "scale", OG_F32);
    require_type(kDq, zp, "zeroPoint", OG_U8);
    if (count < 1) shape(kDq, "count", "count " + std::to_string(count) + " must be at least 1");
    range(kDq, "x", x->length, offset_x, count);
    range(kDq, "y", y->length, offset_y, count);
    range(kDq, "scale", scale->length, offset_scale, 1);
    range(kDq, "zeroPoint", zp->length, offset_zp, 1);
}

// ---- recording ----------------------------------------------------------------------------------------------------

const uint8_t* operand_ptr(const og_operand* o) {
    return o == nullptr ? nullptr
                        : static_cast<const uint8_t*>(o->buffer.ptr) +
                              static_cast<int64_t>(o->offset) * elem_size(o->buffer.type);
}

// Builds the launch description of a validated product.
og::GemmLaunch make_launch(og_int8_gemm* g, const og_int8_gemm_problem* p, const Prepared& pr, const og_buffer* a,
                           const og_buffer* b, const og_operand* za, const og_operand* zb, int out_kind,
                           void* out_base) {
    og::GemmLaunch L = {};
    L.a = static_cast<const uint8_t*>(a->ptr) + p->offset_a;
    L.b = static_cast<const uint8_t*>(b->ptr) + p->offset_b;
    L.m = p->m;
    L.n = p->n;
    L.k = p->k;
    L.batch = p->batch;
    L.trans_b = p->transpose_b != 0;
    L.lda = pr.lda;
    L.ldb = pr.ldb;
    L.stride_a = p->stride_a;
    L.stride_b = p->stride_b;
    L.a_signed = a->type == OG_S8;
    L.b_signed = b->type == OG_S8;
    L.num_sms = g->device->sm_count;
    L.error_flag = g->device->status;
    L.tile = g->tile;
    L.stream_k = g->stream_k;
    og::Epilogue& e = L.epi;
    e.out_kind = out_kind;
    const int esize = out_kind == og::OUT_I32 || out_kind == og::OUT_F32 ? 4 : 1;
    e.c = static_cast<uint8_t*>(out_base) + static_cast<int64_t>(p->offset_c) * esize;
    e.ldc = p->n;
    e.batch_stride_c = static_cast<int64_t>(p->m) * p->n;
    e.m = p->m;
    e.n = p->n;
    e.k = p->k;
    e.za = operand_ptr(za);
    e.za_vector = za ? za->is_vector : 0;
    e.za_signed = a->type == OG_S8;
    e.zb = operand_ptr(zb);
    e.zb_vector = zb ? zb->is_vector : 0;
    e.zb_signed = b->type == OG_S8;
    e.vec_ok = ((reinterpret_cast<uintptr_t>(e.c) & 15) == 0) && ((static_cast<int64_t>(p->n) * esize) % 16 == 0);
    e.sum_splits = 1;
    return L;
}

// Returns device memory for `elements` int32 byte sums from the instance's scratch, growing it geometrically.
int32_t* own_scratch(og_int8_gemm* g, int64_t elements) {
    if (!g->scratch.empty() && g->scratch_elements >= elements) return static_cast<int32_t*>(g->scratch.back());
    int64_t len = std::max<int64_t>(elements, g->scratch.empty() ? 4096 : g->scratch_elements * 2);
    void* p = nullptr;
    check_cuda(cudaMalloc(&p, static_cast<size_t>(len) * sizeof(int32_t)), "Int8Gemm scratch");
    g->scratch.push_back(p);
    g->scratch_elements = len;
    return static_cast<int32_t*>(p);
}

// Chooses the kernel and records the product (and, for the tensor-core path with zero points, the byte sums).
// Device memory for a staged operand (0: A, 1: B) from the instance, growing geometrically.
uint8_t* own_stage(og_int8_gemm* g, int which, int64_t bytes) {
    if (g->stage[which] != nullptr && g->stage_bytes[which] >= bytes) return static_cast<uint8_t*>(g->stage[which]);
    int64_t len = std::max<int64_t>(bytes, std::max<int64_t>(int64_t(1) << 20, g->stage_bytes[which] * 2));
    void* p = nullptr;
    check_cuda(cudaMalloc(&p, static_cast<size_t>(len)), "Int8Gemm staged operand");
    g->scratch.push_back(p);  // freed with the instance
    g->stage[which] = p;
    g->stage_bytes[which] = len;
    return static_cast<uint8_t*>(p);
}

// Copies one operand (`rows` x `width` bytes per batch, `ld` apart, batches `stride` apart) into a pitched buffer of
// the instance whose rows start on 16-byte boundaries, recording the copies; returns the new pitch.
int64_t stage_operand(og_int8_gemm* g, og_encoder* enc, int which, const uint8_t*& base, int64_t ld, int64_t& stride,
                      int batches, int64_t rows, int64_t width) {
    const int64_t pitch = (width + 15) & ~int64_t(15);
    uint8_t* dst = own_stage(g, which, batches * rows * pitch);
    const uint8_t* src = base;
    const int64_t sstride = stride;
    if (batches == 1 || sstride == rows * ld) {
        // One two-dimensional copy covers every batch (shared, or dense batches).
        const int64_t height = (batches == 1 ? 1 : batches) * rows;
        enc->ops.push_back([=](cudaStream_t s) {
            return cudaMemcpy2DAsync(dst, static_cast<size_t>(pitch), src, static_cast<size_t>(ld),
                                     static_cast<size_t>(width), static_cast<size_t>(height), cudaMemcpyDeviceToDevice,
                                     s);
        });
    } else {
        enc->ops.push_back([=](cudaStream_t s) {
            for (int b = 0; b < batches; b++) {
                const cudaError_t e = cudaMemcpy2DAsync(dst + b * rows * pitch, static_cast<size_t>(pitch),
                                                        src + b * sstride, static_cast<size_t>(ld),
                                                        static_cast<size_t>(width), static_cast<size_t>(rows),
                                                        cudaMemcpyDeviceToDevice, s);
                if (e != cudaSuccess) return e;
            }
            return cudaSuccess;
        });
    }
    base = dst;
    stride = batches > 1 ? rows * pitch : 0;
    return pitch;
}

// Products large enough for the tensor cores whose A or B rows (or batches) do not start on 16-byte boundaries, so
// that TMA cannot load them in place: the misaligned operand is copied into a pitched buffer (rows padded to 16 bytes;
// the padding is never read) and the tensor-core product runs on the copy. The copy moves each operand byte once;
// the portable kernel it replaces runs far below the tensor cores' rate at these sizes.
constexpr int64_t kStageMinOps = int64_t(1) << 27;

bool stage_for_tensor_cores(og_int8_gemm* g, og_encoder* enc, og::GemmLaunch& L) {
    if (L.k < 1 || L.m < 1 || L.n < 1 || 2.0 * L.m * L.n * L.k * L.batch < double(kStageMinOps)) return false;
    auto misaligned = [](const uint8_t* p, int64_t ld, int64_t stride, int batches) {
        return (reinterpret_cast<uintptr_t>(p) & 15) != 0 || (ld & 15) != 0 || (batches > 1 && (stride & 15) != 0);
    };
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    bool staged = false;
    if (misaligned(L.a, L.lda, L.stride_a, ba)) {
        L.lda = stage_operand(g, enc, 0, L.a, L.lda, L.stride_a, ba, L.m, L.k);
        staged = true;
    }
    if (misaligned(L.b, L.ldb, L.stride_b, bb)) {
        const int64_t rows = L.trans_b ? L.n : L.k, width = L.trans_b ? L.k : L.n;
        L.ldb = stage_operand(g, enc, 1, L.b, L.ldb, L.stride_b, bb, rows, width);
        staged = true;
    }
    return staged;
}

void record_gemm(og_int8_gemm* g, og_encoder* enc, og::GemmLaunch L, const og_operand* caller_scratch) {
    const bool want_tc = g->allow_dot && g->kernel != OG_KERNEL_PORTABLE;
    bool tc = want_tc && og::tc_eligible(L);
    bool staged = false;
    if (want_tc && !tc && g->kernel == OG_KERNEL_AUTO) {
        staged = stage_for_tensor_cores(g, enc, L);
        tc = staged && og::tc_eligible(L);
    }
    if (g->kernel == OG_KERNEL_TENSOR_CORE && !tc) {
        unsupported(kGemm,
                    "the tensor-core kernel needs K >= 1 and operands whose rows and batches start on 16-byte "
                    "boundaries",
                    "TensorCoreInt8", "16-byte aligned operands", "unaligned operand or K = 0");
    }
    if (tc && g->kernel == OG_KERNEL_AUTO && static_cast<int64_t>(L.m) * L.n * L.k < (int64_t(1) << 16)) tc = false;
    if (!tc) {
        g->last = "portable";
        enc->ops.push_back([L](cudaStream_t s) { return og::launch_gemm_simt(L, s); });
        enc->dispatches += 1;
        return;
    }
    if (g->tile == 0 && og::rows_eligible(L)) {
        const int workers = og::rows_workers(L);
        if (workers > 0) {
            // Partials and tickets of the even split, owned by the instance (tickets start at zero and every launch
            // leaves them there); recorded launches of one instance run in stream order, so they share them.
            const int64_t part = og::rows_part_ints(L, workers), tickets = og::rows_tickets(L);
            if (g->rows_part_ints < part || g->rows_ticket_count < tickets) {
                void* pp = nullptr;
                void* tp = nullptr;
                check_cuda(cudaMalloc(&pp, static_cast<size_t>(part) * sizeof(int32_t)), "Int8Gemm split partials");
                g->rows_bufs.push_back(pp);
                check_cuda(cudaMalloc(&tp, static_cast<size_t>(tickets) * sizeof(unsigned int)), "Int8Gemm tickets");
                g->rows_bufs.push_back(tp);
                check_cuda(cudaMemset(tp, 0, static_cast<size_t>(tickets) * sizeof(unsigned int)), "Int8Gemm tickets");
                g->rows_part = static_cast<int32_t*>(pp);
                g->rows_ticket = static_cast<unsigned int*>(tp);
                g->rows_part_ints = part;
                g->rows_ticket_count = tickets;
            }
            L.rows_part = g->rows_part;
            L.rows_ticket = g->rows_ticket;
            L.rows_workers = workers;
        }
        cudaError_t err;
        og::LaunchFn fn = og::prepare_gemm_rows(L, &err);  // tensor maps built now, at record time
        check_cuda(err, "Int8Gemm tensor maps");
        g->last = staged ? "tensor-core-rows-staged" : "tensor-core-rows";
        enc->ops.push_back(std::move(fn));
        enc->dispatches += 1;
        return;
    }
    const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
    const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
    const bool need_rows = L.epi.zb != nullptr;  // zb * rowsum(A)
    const bool need_cols = L.epi.za != nullptr;  // za * colsum(B)
    int32_t* rows = nullptr;
    int32_t* cols = nullptr;
    if (need_rows || need_cols) {
        // Up to 8 partial sums over K per row / column, so that the sums pass has enough CTAs (see byte_sum_splits).
        const int splits = og::byte_sum_splits(L, 8);
        const int64_t row_elems = need_rows ? int64_t(ba) * L.m : 0;
        const int64_t col_elems = need_cols ? int64_t(bb) * L.n : 0;
        const int64_t need = splits * (row_elems + col_elems);
        int32_t* base = nullptr;
        if (caller_scratch != nullptr &&
            caller_scratch->buffer.length - caller_scratch->offset >= need)
            base = static_cast<int32_t*>(caller_scratch->buffer.ptr) + caller_scratch->offset;
        else
            base = own_scratch(g, need);
        rows = need_rows ? base : nullptr;
        cols = need_cols ? base + splits * row_elems : nullptr;
        L.epi.row_sum_a = rows;
        L.epi.row_sum_a_stride = ba > 1 ? L.m : 0;
        L.epi.col_sum_b = cols;
        L.epi.col_sum_b_stride = bb > 1 ? L.n : 0;
        L.epi.sum_splits = splits;
        L.epi.row_sum_split_stride = row_elems;
        L.epi.col_sum_split_stride = col_elems;
        cudaError_t err;
        og::LaunchFn sums = og::prepare_byte_sums(L, rows, cols, splits, &err);
        check_cuda(err, "Int8Gemm byte sums");
        enc->ops.push_back(std::move(sums));
        enc->dispatches += 1;
    }
    const int split = og::tc_split_mode(L);
    if (split != 0) {
        // Products whose last wave of tiles would leave SMs idle split some of the (tile, K block) work across the
        // workers; split tiles meet through this buffer. Recorded launches of one instance run in stream order, so
        // they share it.
        if (g->sk_buf == nullptr) {
            const int64_t bytes = og::sk_bytes_needed(L.num_sms);
            check_cuda(cudaMalloc(&g->sk_buf, static_cast<size_t>(bytes)), "Int8Gemm stream-K buffer");
            check_cuda(cudaMemset(g->sk_buf, 0, static_cast<size_t>(bytes)), "Int8Gemm stream-K buffer");
            g->sk_bytes = bytes;
        }
        og::sk_bind(L, g->sk_buf, g->sk_bytes);
    }
    cudaError_t err;
    og::LaunchFn fn = og::prepare_gemm_tc(L, &err);  // tensor maps built now, at record time
    check_cuda(err, "Int8Gemm tensor maps");
    g->last = std::string(og::tc_cta_group(L) == 2 ? "tensor-core-2sm" : "tensor-core-1sm") +
              (split == 2 ? "-stream-k" : split == 1 ? "-split-tail" : "") + (staged ? "-staged" : "");
    enc->ops.push_back(std::move(fn));
    enc->dispatches += 1;
}

og_int8_gemm* live_gemm(og_int8_gemm* g) {
    if (g == nullptr) throw OgError{OG_ERROR_INVALID_HANDLE, kGemm, "gemm", "null Int8Gemm handle", "", "", ""};
    return g;
}

}  // namespace

// ---- C ABI --------------------------------------------------------------------------------------------------------

extern "C" {

OG_API og_status og_last_error(og_error_info* out) {
    if (out == nullptr) return OG_ERROR_ARGUMENT_NULL;
    *out = g_last;
    return OG_OK;
}

OG_API og_status og_device_count(int32_t* count) {
    return guard([&] {
        if (count == nullptr) null_arg("GpuDevice", "count");
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
            cudaGetLastError();
            n = 0;
        } else {
            check_cuda(e, "cudaGetDeviceCount");
        }
        *count = n;
    });
}

OG_API og_status og_device_create(int32_t ordinal, og_device** out) {
    return guard([&] {
        if (out == nullptr) null_arg("GpuDevice", "out");
        *out = nullptr;
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || ordinal < 0 || ordinal >= n) {
            cudaGetLastError();
            unsupported("GpuDevice", "no CUDA device " + std::to_string(ordinal), "Device",
                        "a CUDA device ordinal below " + std::to_string(n), std::to_string(ordinal));
        }
        auto* d = new og_device();
        d->ordinal = ordinal;
        try {
            use(d);
            check_cuda(cudaGetDeviceProperties(&d->prop, ordinal), "cudaGetDeviceProperties");
            d->sm_count = d->prop.multiProcessorCount;
            check_cuda(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "cudaStreamCreate");
            check_cuda(cudaStreamCreateWithFlags(&d->upload, cudaStreamNonBlocking), "cudaStreamCreate");
            check_cuda(cudaStreamCreateWithFlags(&d->readback, cudaStreamNonBlocking), "cudaStreamCreate");
            check_cuda(cudaMalloc(&d->status, sizeof(int)), "cudaMalloc");
            check_cuda(cudaMemset(d->status, 0, sizeof(int)), "cudaMemset");
            check_cuda(cudaMallocHost(&d->status_host, sizeof(int)), "cudaMallocHost");
            check_cuda(cudaMallocHost(&d->readback_words, kReadbackWords * sizeof(int)), "cudaMallocHost");
            d->readback_free.reserve(kReadbackWords);
            for (int i = kReadbackWords - 1; i >= 0; i--) d->readback_free.push_back(i);
        } catch (...) {
            if (d->stream) cudaStreamDestroy(d->stream);
            if (d->upload) cudaStreamDestroy(d->upload);
            if (d->readback) cudaStreamDestroy(d->readback);
            if (d->status) cudaFree(d->status);
            if (d->status_host) cudaFreeHost(d->status_host);
            delete d;
            throw;
        }
        *out = d;
    });
}

OG_API og_status og_device_destroy(og_device* d) {
    return guard([&] {
        if (d == nullptr) return;
        use(d);
        cudaStreamSynchronize(d->stream);
        cudaStreamSynchronize(d->upload);
        cudaStreamSynchronize(d->readback);
        if (d->own_stream) cudaStreamDestroy(d->stream);
        cudaStreamDestroy(d->upload);
        cudaStreamDestroy(d->readback);
        cudaFree(d->status);
        cudaFreeHost(d->status_host);
        cudaFreeHost(d->readback_words);
        delete d;
    });
}

OG_API og_status og_device_info_get(og_device* d, og_device_info* out) {
    return guard([&] {
        if (d == nullptr || out == nullptr) null_arg("GpuDevice", "device");
        og_device_info i = {};
        copy_field(i.name, sizeof(i.name), d->prop.name);
        i.ordinal = d->ordinal;
        i.sm_count = d->sm_count;
        i.cc_major = d->prop.major;
        i.cc_minor = d->prop.minor;
        i.total_memory = static_cast<int64_t>(d->prop.totalGlobalMem);
        i.max_shared_memory_per_block = static_cast<int32_t>(d->prop.sharedMemPerBlockOptin);
        i.tensor_core_i8 = d->prop.major == 10 && d->prop.minor == 0;
        *out = i;
    });
}

OG_API og_status og_device_wait_idle(og_device* d) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        use(d);
        check_cuda(cudaStreamSynchronize(d->upload), "WaitIdle");
        check_cuda(cudaStreamSynchronize(d->readback), "WaitIdle");
        check_device_status(d);
    });
}

namespace og {
// One thread waits, with the kernels' own bounded wait, on an mbarrier that expects an arrival nobody makes. The wait
// gives up after limit_ns, the kernel raises the device's failure word the way a stalled product kernel does, and it
// returns: no fault, no trap, nothing left in flight.
__global__ void watchdog_selftest_kernel(int* status, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x != 0) return;
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (!mbar_wait(&bar, 0, &abort_flag, limit_ns)) atomicExch(status, 1);
}
}  // namespace og

OG_API og_status og_device_watchdog_selftest(og_device* d, uint32_t limit_us) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (limit_us < 1 || limit_us > 2000000)
            throw OgError{OG_ERROR_ARGUMENT_RANGE, "GpuDevice", "limitMicroseconds",
                          "the self-test wait limit is 1 .. 2000000 microseconds", "", "", ""};
        use(d);
        og::watchdog_selftest_kernel<<<1, 32, 0, d->stream>>>(d->status, uint64_t(limit_us) * 1000);
        check_cuda(cudaGetLastError(), "watchdog self-test launch");
    });
}

OG_API og_status og_device_stream(og_device* d, void** stream) {
    return guard([&] {
        if (d == nullptr || stream == nullptr) null_arg("GpuDevice", "device");
        *stream = d->stream;
    });
}

OG_API og_status og_device_set_stream(og_device* d, void* stream) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        use(d);
        check_cuda(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
        if (d->own_stream) cudaStreamDestroy(d->stream);
        d->stream = static_cast<cudaStream_t>(stream);
        d->own_stream = false;
    });
}

OG_API og_status og_buffer_alloc(og_device* d, uint64_t bytes, void** ptr) {
    return guard([&] {
        if (d == nullptr || ptr == nullptr) null_arg("GpuDevice", "device");
        use(d);
        *ptr = nullptr;
        check_cuda(cudaMallocAsync(ptr, bytes == 0 ? 16 : bytes, d->stream), "CreateBuffer");
        check_cuda(cudaStreamSynchronize(d->stream), "CreateBuffer");
    });
}

OG_API og_status og_buffer_free(og_device* d, void* ptr) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (ptr == nullptr) return;
        use(d);
        check_cuda(cudaFreeAsync(ptr, d->stream), "GpuBuffer.Dispose");
    });
}

OG_API og_status og_buffer_write(og_device* d, void* dst, const void* src, uint64_t bytes) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (bytes == 0) return;
        if (dst == nullptr || src == nullptr) null_arg("GpuDevice", "buffer");
        use(d);
        check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, d->stream), "WriteBuffer");
    });
}

OG_API og_status og_buffer_read(og_device* d, void* dst, const void* src, uint64_t bytes) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (dst == nullptr || src == nullptr) null_arg("GpuDevice", "buffer");
        use(d);
        if (bytes != 0) check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, d->stream), "ReadAsync");
        check_device_status(d);
    });
}

OG_API og_status og_buffer_write_async(og_device* d, void* dst, const void* src, uint64_t bytes) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (bytes == 0) return;
        if (dst == nullptr || src == nullptr) null_arg("GpuDevice", "buffer");
        use(d);
        cudaEvent_t done = nullptr;
        check_cuda(cudaEventCreateWithFlags(&done, cudaEventDisableTiming), "WriteBuffer");
        cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, d->upload);
        if (e == cudaSuccess) e = cudaEventRecord(done, d->upload);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(d->stream, done, 0);  // later submissions wait for the upload
        cudaEventDestroy(done);
        check_cuda(e, "WriteBuffer");
    });
}

OG_API og_status og_buffer_read_async(og_device* d, void* dst, const void* src, uint64_t bytes, og_readback** out) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (out == nullptr) null_arg("GpuDevice", "readback");
        if (dst == nullptr || src == nullptr) null_arg("GpuDevice", "buffer");
        use(d);
        auto* r = new og_readback();
        r->device = d;
        try {
            cudaEvent_t submitted = nullptr;
            take_status_word(d, r);
            check_cuda(cudaEventCreateWithFlags(&submitted, cudaEventDisableTiming), "ReadAsync");
            cudaError_t e = cudaEventRecord(submitted, d->stream);  // everything submitted so far
            if (e == cudaSuccess) e = cudaStreamWaitEvent(d->readback, submitted, 0);
            cudaEventDestroy(submitted);
            check_cuda(e, "ReadAsync");
            check_cuda(cudaMemcpyAsync(r->status_host, d->status, sizeof(int), cudaMemcpyDeviceToHost, d->readback),
                       "ReadAsync");
            if (bytes != 0)
                check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, d->readback), "ReadAsync");
            check_cuda(cudaEventCreateWithFlags(&r->done, cudaEventDisableTiming), "ReadAsync");
            check_cuda(cudaEventRecord(r->done, d->readback), "ReadAsync");
        } catch (...) {
            if (r->done) cudaEventDestroy(r->done);
            give_status_word(r);
            delete r;
            throw;
        }
        *out = r;
    });
}

OG_API og_status og_readback_wait(og_readback* r) {
    return guard([&] {
        if (r == nullptr) null_arg("GpuDevice", "readback");
        struct Release {
            og_readback* r;
            ~Release() {
                cudaEventDestroy(r->done);
                give_status_word(r);
                delete r;
            }
        } release{r};
        use(r->device);
        check_cuda(cudaEventSynchronize(r->done), "ReadAsync");
        if (*r->status_host != 0)
            throw OgError{OG_ERROR_COMMAND_FAILED, "GpuDevice", "",
                          "a kernel gave up waiting on its own pipeline (watchdog) and skipped its work", "Watchdog",
                          "", ""};
    });
}

OG_API og_status og_buffer_fill(og_device* d, void* dst, int32_t value, uint64_t bytes) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (bytes == 0) return;
        if (dst == nullptr) null_arg("GpuDevice", "buffer");
        use(d);
        check_cuda(cudaMemsetAsync(dst, value, bytes, d->stream), "fill");
    });
}

OG_API og_status og_host_alloc(uint64_t bytes, void** ptr) {
    return guard([&] {
        if (ptr == nullptr) null_arg("host", "ptr");
        check_cuda(cudaMallocHost(ptr, bytes == 0 ? 16 : bytes), "cudaMallocHost");
    });
}

OG_API og_status og_host_free(void* ptr) {
    return guard([&] {
        if (ptr != nullptr) check_cuda(cudaFreeHost(ptr), "cudaFreeHost");
    });
}

OG_API og_status og_encoder_begin(og_device* d, og_encoder** out) {
    return guard([&] {
        if (d == nullptr || out == nullptr) null_arg("GpuDevice", "device");
        auto* e = new og_encoder();
        e->device = d;
        *out = e;
    });
}

OG_API og_status og_encoder_discard(og_encoder* e) {
    delete e;
    return OG_OK;
}

OG_API og_status og_encoder_dispatch_count(og_encoder* e, int64_t* count) {
    return guard([&] {
        if (e == nullptr || count == nullptr) null_arg("GpuCommandEncoder", "encoder");
        *count = e->dispatches;
    });
}

OG_API og_status og_device_submit(og_device* d, og_encoder* e) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (e == nullptr) null_arg("GpuDevice", "encoder");
        struct Consume {
            og_encoder* e;
            ~Consume() { delete e; }
        } consume{e};
        if (e->device != d)
            throw OgError{OG_ERROR_INVALID_HANDLE, "GpuDevice", "encoder", "the encoder belongs to another device",
                          "", "", ""};
        use(d);
        for (auto& op : e->ops) check_cuda(op(d->stream), "Submit");
    });
}

OG_API og_status og_device_capture_begin(og_device* d) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        use(d);
        check_cuda(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeRelaxed), "BeginCapture");
    });
}

OG_API og_status og_device_capture_end(og_device* d, og_graph** out) {
    return guard([&] {
        if (d == nullptr) null_arg("GpuDevice", "device");
        if (out == nullptr) null_arg("GpuDevice", "out");
        use(d);
        cudaGraph_t graph = nullptr;
        check_cuda(cudaStreamEndCapture(d->stream, &graph), "EndCapture");
        cudaGraphExec_t exec = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
        if (e != cudaSuccess) {
            cudaGraphDestroy(graph);
            check_cuda(e, "EndCapture");
        }
        auto* g = new og_graph();
        g->device = d;
        g->graph = graph;
        g->exec = exec;
        *out = g;
    });
}

OG_API og_status og_graph_launch(og_graph* g) {
    return guard([&] {
        if (g == nullptr) null_arg("GpuGraph", "graph");
        use(g->device);
        check_cuda(cudaGraphLaunch(g->exec, g->device->stream), "GraphLaunch");
    });
}

OG_API og_status og_graph_destroy(og_graph* g) {
    return guard([&] {
        if (g == nullptr) return;
        use(g->device);
        cudaStreamSynchronize(g->device->stream);
        cudaGraphExecDestroy(g->exec);
        cudaGraphDestroy(g->graph);
        delete g;
    });
}

OG_API og_status og_timestamps_create(og_device* d, uint32_t count, og_timestamps** out) {
    return guard([&] {
        if (d == nullptr || out == nullptr) null_arg("GpuDevice", "device");
        use(d);
        auto* t = new og_timestamps();
        t->device = d;
        t->events.resize(count, nullptr);
        for (auto& ev : t->events) check_cuda(cudaEventCreate(&ev), "CreateTimestampSet");
        *out = t;
    });
}

OG_API og_status og_timestamps_destroy(og_timestamps* t) {
    return guard([&] {
        if (t == nullptr) return;
        use(t->device);
        for (auto ev : t->events)
            if (ev) cudaEventDestroy(ev);
        delete t;
    });
}

OG_API og_status og_encoder_timestamp(og_encoder* e, og_timestamps* t, uint32_t index) {
    return guard([&] {
        if (e == nullptr || t == nullptr) null_arg("GpuCommandEncoder", "timestamps");
        if (index >= t->events.size())
            throw OgError{OG_ERROR_ARGUMENT_RANGE, "GpuCommandEncoder", "index", "timestamp index out of range", "",
                          "", ""};
        cudaEvent_t ev = t->events[index];
        e->ops.push_back([ev](cudaStream_t s) { return cudaEventRecord(ev, s); });
    });
}

OG_API og_status og_device_timestamp(og_device* d, og_timestamps* t, uint32_t index) {
    return guard([&] {
        if (d == nullptr || t == nullptr) null_arg("GpuDevice", "timestamps");
        if (index >= t->events.size())
            throw OgError{OG_ERROR_ARGUMENT_RANGE, "GpuDevice", "index", "timestamp index out of range", "", "", ""};
        use(d);
        check_cuda(cudaEventRecord(t->events[index], d->stream), "timestamp");
    });
}

OG_API og_status og_timestamps_read(og_timestamps* t, uint32_t first, uint32_t count, double* ns) {
    return guard([&] {
        if (t == nullptr || ns == nullptr) null_arg("GpuDevice", "timestamps");
        if (static_cast<uint64_t>(first) + count > t->events.size())
            throw OgError{OG_ERROR_ARGUMENT_RANGE, "GpuDevice", "first", "timestamp range out of range", "", "", ""};
        use(t->device);
        for (uint32_t i = 0; i < count; i++) {
            check_cuda(cudaEventSynchronize(t->events[first + i]), "TryReadTimestamps");
            float ms = 0.0f;
            check_cuda(cudaEventElapsedTime(&ms, t->events[first], t->events[first + i]), "TryReadTimestamps");
            ns[i] = static_cast<double>(ms) * 1e6;
        }
    });
}

// ---- Int8Gemm -------------------------------------------------------------------------------------------------------

OG_API og_status og_int8_gemm_create(og_device* d, const og_int8_gemm_options* options, og_int8_gemm** out) {
    return guard([&] {
        if (d == nullptr) null_arg(kGemm, "device");
        if (out == nullptr) null_arg(kGemm, "out");
        auto* g = new og_int8_gemm();
        g->device = d;
        g->allow_dot = options == nullptr || options->allow_packed_dot != 0;
        g->kernel = options == nullptr ? OG_KERNEL_AUTO : options->kernel;
        g->tile = options == nullptr ? 0 : options->tile;
        g->stream_k = options == nullptr ? 0 : options->stream_k;
        if (g->stream_k < 0 || g->stream_k > 2)
            throw OgError{OG_ERROR_ARGUMENT_RANGE, kGemm, "StreamK", "the stream-K hook takes 0, 1 or 2", "", "", ""};
        if (g->tile != 0 && g->tile != 128 && g->tile != 256) {
            delete g;
            throw OgError{OG_ERROR_ARGUMENT_RANGE, kGemm, "Tile", "the tile hook takes 0, 128 or 256", "", "", ""};
        }
        const bool tc_hw = d->prop.major == 10 && d->prop.minor == 0;
        if (g->kernel == OG_KERNEL_TENSOR_CORE && (!tc_hw || !g->allow_dot)) {
            delete g;
            unsupported(kGemm, "the tcgen05 int8 kernel needs an sm_100 device", "TensorCoreInt8", "sm_100",
                        "sm_" + std::to_string(d->prop.major) + std::to_string(d->prop.minor));
        }
        if (!tc_hw) g->allow_dot = false;
        const char* tcv = g->tile == 128   ? "tcgen05-i8-1sm-tile128x256x128"
                          : g->tile == 256 ? "tcgen05-i8-2sm-tile256x256x128"
                                           : "tcgen05-i8-2sm-tile256x256x128+1sm-tile128x256x128";
        g->variant = g->allow_dot && g->kernel != OG_KERNEL_PORTABLE ? tcv : "portable-simt-tile64x64x32";
        *out = g;
    });
}

OG_API og_status og_int8_gemm_destroy(og_int8_gemm* g) {
    return guard([&] {
        if (g == nullptr) return;
        use(g->device);
        cudaStreamSynchronize(g->device->stream);
        for (void* p : g->scratch) cudaFree(p);
        for (void* p : g->rows_bufs) cudaFree(p);
        if (g->sk_buf != nullptr) cudaFree(g->sk_buf);
        delete g;
    });
}

OG_API og_status og_int8_gemm_variant(og_int8_gemm* g, char* buffer, uint64_t capacity) {
    return guard([&] { put_string(buffer, capacity, live_gemm(g)->variant); });
}

OG_API og_status og_int8_gemm_last_kernel(og_int8_gemm* g, char* buffer, uint64_t capacity) {
    return guard([&] { put_string(buffer, capacity, live_gemm(g)->last); });
}

OG_API int64_t og_int8_gemm_scratch_elements(const og_int8_gemm_problem* p) {
    if (p == nullptr || p->m <= 0 || p->n <= 0 || p->batch <= 0) return 0;
    return static_cast<int64_t>(p->batch) * p->m * p->n;
}

OG_API og_status og_int8_gemm_reserve_scratch(og_int8_gemm* g, int64_t elements) {
    return guard([&] {
        live_gemm(g);
        if (elements < 0 || elements > kMaxElements)
            throw OgError{OG_ERROR_ARGUMENT_RANGE, kGemm, "elements",
                          "must be between 0 and " + std::to_string(kMaxElements), "", "", ""};
        if (elements == 0 || (!g->scratch.empty() && g->scratch_elements >= elements)) return;
        use(g->device);
        own_scratch(g, std::max<int64_t>(elements, 4096));
    });
}

OG_API og_status og_int8_gemm_bind_groups_created(og_int8_gemm* g, int32_t* count) {
    return guard([&] {
        live_gemm(g);
        if (count == nullptr) null_arg(kGemm, "count");
        *count = 0;
    });
}

OG_API og_status og_int8_gemm_check_int32(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b,
                                          const og_buffer* c, const og_operand* za, const og_operand* zb,
                                          const og_operand* bias) {
    return guard([&] { check_int32(p, a, b, c, za, zb, bias); });
}

OG_API og_status og_int8_gemm_check_float(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b,
                                          const og_buffer* c, const og_operand* scale, const og_operand* za,
                                          const og_operand* zb, const og_operand* fbias, const og_operand* ibias) {
    return guard([&] { check_float(p, a, b, c, scale, za, zb, fbias, ibias); });
}

OG_API og_status og_int8_gemm_check_requantized(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b,
                                                const og_buffer* y, const og_operand* mult, int32_t zero_y,
                                                const og_operand* za, const og_operand* zb, const og_operand* ibias,
                                                const og_operand* scratch) {
    return guard([&] { check_requantized(p, a, b, y, mult, zero_y, za, zb, ibias, scratch); });
}

OG_API og_status og_int8_gemm_encode_int32(og_int8_gemm* g, og_encoder* enc, const og_int8_gemm_problem* p,
                                           const og_buffer* a, const og_buffer* b, const og_buffer* c,
                                           const og_operand* za, const og_operand* zb, const og_operand* bias) {
    return guard([&] {
        live_gemm(g);
        if (c == nullptr || c->ptr == nullptr) null_arg(kGemm, "c");
        if (enc == nullptr) null_arg(kGemm, "encoder");
        const Prepared pr = check_int32(p, a, b, c, za, zb, bias);
        if (!pr.ok) {
            g->last = "none";
            return;
        }
        use(g->device);
        og::GemmLaunch L = make_launch(g, p, pr, a, b, za, zb, og::OUT_I32, c->ptr);
        L.epi.int_bias = reinterpret_cast<const int32_t*>(operand_ptr(bias));
        record_gemm(g, enc, L, nullptr);
    });
}

OG_API og_status og_int8_gemm_encode_float(og_int8_gemm* g, og_encoder* enc, const og_int8_gemm_problem* p,
                                           const og_buffer* a, const og_buffer* b, const og_buffer* c,
                                           const og_operand* scale, const og_operand* za, const og_operand* zb,
                                           const og_operand* fbias, const og_operand* ibias) {
    return guard([&] {
        live_gemm(g);
        if (c == nullptr || c->ptr == nullptr) null_arg(kGemm, "c");
        if (enc == nullptr) null_arg(kGemm, "encoder");
        const Prepared pr = check_float(p, a, b, c, scale, za, zb, fbias, ibias);
        if (!pr.ok) {
            g->last = "none";
            return;
        }
        use(g->device);
        og::GemmLaunch L = make_launch(g, p, pr, a, b, za, zb, og::OUT_F32, c->ptr);
        L.epi.int_bias = reinterpret_cast<const int32_t*>(operand_ptr(ibias));
        L.epi.scale = reinterpret_cast<const float*>(operand_ptr(scale));
        L.epi.scale_vector = scale->is_vector;
        L.epi.float_bias = reinterpret_cast<const float*>(operand_ptr(fbias));
        record_gemm(g, enc, L, nullptr);
    });
}

OG_API og_status og_int8_gemm_check_dequantize(const og_int8_gemm_problem* p, const og_buffer* a, const og_buffer* b,
                                               const og_buffer* c, const og_operand* a_scale, const og_operand* b_scale,
                                               const og_operand* za, const og_operand* zb, const og_operand* fbias,
                                               const og_operand* ibias) {
    return guard([&] { check_dequantize(p, a, b, c, a_scale, b_scale, za, zb, fbias, ibias); });
}

OG_API og_status og_int8_gemm_encode_dequantize(og_int8_gemm* g, og_encoder* enc, const og_int8_gemm_problem* p,
                                                const og_buffer* a, const og_buffer* b, const og_buffer* c,
                                                const og_operand* a_scale, const og_operand* b_scale,
                                                const og_operand* za, const og_operand* zb, const og_operand* fbias,
                                                const og_operand* ibias) {
    return guard([&] {
        live_gemm(g);
        if (c == nullptr || c->ptr == nullptr) null_arg(kGemm, "c");
        if (enc == nullptr) null_arg(kGemm, "encoder");
        const Prepared pr = check_dequantize(p, a, b, c, a_scale, b_scale, za, zb, fbias, ibias);
        if (!pr.ok) {
            g->last = "none";
            return;
        }
        use(g->device);
        og::GemmLaunch L = make_launch(g, p, pr, a, b, za, zb, og::OUT_F32, c->ptr);
        L.epi.int_bias = reinterpret_cast<const int32_t*>(operand_ptr(ibias));
        L.epi.scale = reinterpret_cast<const float*>(operand_ptr(b_scale));
        L.epi.scale_vector = b_scale->is_vector;
        L.epi.scale_a = reinterpret_cast<const float*>(operand_ptr(a_scale));
        L.epi.float_bias = reinterpret_cast<const float*>(operand_ptr(fbias));
        record_gemm(g, enc, L, nullptr);
    });
}

OG_API og_status og_int8_gemm_encode_requantized(og_int8_gemm* g, og_encoder* enc, const og_int8_gemm_problem* p,
                                                 const og_buffer* a, const og_buffer* b, const og_buffer* y,
                                                 const og_operand* mult, int32_t zero_y, const og_operand* za,
                                                 const og_operand* zb, const og_operand* ibias,
                                                 const og_operand* scratch) {
    return guard([&] {
        live_gemm(g);
        if (y == nullptr || y->ptr == nullptr) null_arg(kGemm, "y");
        if (enc == nullptr) null_arg(kGemm, "encoder");
        const Prepared pr = check_requantized(p, a, b, y, mult, zero_y, za, zb, ibias, scratch);
        if (!pr.ok) {
            g->last = "none";
            return;
        }
        use(g->device);
        og::GemmLaunch L =
            make_launch(g, p, pr, a, b, za, zb, y->type == OG_U8 ? og::OUT_U8 : og::OUT_S8, y->ptr);
        L.epi.int_bias = reinterpret_cast<const int32_t*>(operand_ptr(ibias));
        L.epi.scale = reinterpret_cast<const float*>(operand_ptr(mult));
        L.epi.scale_vector = mult->is_vector;
        L.epi.zero_point_y = zero_y;
        record_gemm(g, enc, L, scratch);
    });
}

// ---- DynamicQuantizeKernels -----------------------------------------------------------------------------------------

OG_API og_status og_dynamic_quantize_create(og_device* d, og_dynamic_quantize** out) {
    return guard([&] {
        if (d == nullptr) null_arg(kDq, "device");
        if (out == nullptr) null_arg(kDq, "out");
        use(d);
        auto* q = new og_dynamic_quantize();
        q->device = d;
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, og::dq_scratch_bytes());
        if (e != cudaSuccess) {
            delete q;
            check_cuda(e, "dynamic quantize ranges");
        }
        check_cuda(cudaMemset(p, 0, og::dq_scratch_bytes()), "dynamic quantize ranges");
        q->scratch = static_cast<og::DqScratch*>(p);
        *out = q;
    });
}

OG_API og_status og_dynamic_quantize_destroy(og_dynamic_quantize* q) {
    return guard([&] {
        if (q == nullptr) return;
        use(q->device);
        cudaStreamSynchronize(q->device->stream);
        cudaFree(q->scratch);
        delete q;
    });
}

OG_API og_status og_dynamic_quantize_check(const og_buffer* x, int32_t offset_x, int32_t count, const og_buffer* y,
                                           int32_t offset_y, const og_buffer* scale, int32_t offset_scale,
                                           const og_buffer* zp, int32_t offset_zp) {
    return guard([&] { check_dq(x, offset_x, count, y, offset_y, scale, offset_scale, zp, offset_zp); });
}

OG_API og_status og_dynamic_quantize_encode(og_dynamic_quantize* q, og_encoder* enc, const og_buffer* x,
                                            int32_t offset_x, int32_t count, const og_buffer* y, int32_t offset_y,
                                            const og_buffer* scale, int32_t offset_scale, const og_buffer* zp,
                                            int32_t offset_zp) {
    return guard([&] {
        if (q == nullptr) throw OgError{OG_ERROR_INVALID_HANDLE, kDq, "dq", "null handle", "", "", ""};
        if (enc == nullptr) null_arg(kDq, "encoder");
        check_dq(x, offset_x, count, y, offset_y, scale, offset_scale, zp, offset_zp);
        use(q->device);
        const float* xp = static_cast<const float*>(x->ptr) + offset_x;
        uint8_t* yp = static_cast<uint8_t*>(y->ptr) + offset_y;
        float* sp = static_cast<float*>(scale->ptr) + offset_scale;
        uint8_t* zpp = static_cast<uint8_t*>(zp->ptr) + offset_zp;
        og::DqScratch* scr = q->scratch;
        const int sms = q->device->sm_count;
        int* status = q->device->status;
        const int64_t n = count;
        enc->ops.push_back(
            [=](cudaStream_t s) { return og::launch_dynamic_quantize(xp, n, yp, sp, zpp, scr, sms, status, s); });
        enc->dispatches += og::dq_single_kernel(xp, n, yp) ? 1 : 2;
    });
}

}  // extern "C"

// ---- EncodeInt32 without allocation ---------------------------------------------------------------------------------
//
// Some callers cannot call cudaMalloc while they run products: serving hosts that reserve all of a GPU's memory for
// their own pool at start-up (any other allocation fails or eats into the pool), engines whose execution step only
// hands a kernel pre-sized workspaces and forbids allocation inside it, and latency-bound loops (a decode step) that
// cannot afford cudaMalloc's implicit device synchronisation. Int8Gemm allocates (and grows) the scratch of the byte
// sums that the zero-point correction needs on its first products, so such callers get og_int8_gemm_int32_noalloc
// instead: the same product, the same checks, the same kernels, with the byte sums kept in a fixed array of device
// memory that is part of this library.
//
// The array holds at most kNoAllocSumElements int32 sums (row sums of A for every batch of A when B has a zero point,
// plus column sums of B for every batch of B when A has one); larger requests are refused. Every GPU that loads the
// library keeps the array (4 MiB) until the process exits. All calls share it and it keeps the last call's contents:
// the column sums, which are accumulated with atomics, are cleared on the stream before each use, and calls whose
// work overlaps on the GPU (different streams, no ordering between them) race on it.
//
// The kernels of these calls report a bounded wait that gave up through the word g_noalloc_status of the device,
// not through an og_device: og_int8_gemm_noalloc_status reads it back on the caller's stream and clears it.

namespace {

constexpr int64_t kNoAllocSumElements = int64_t(1) << 20;

static __device__ __align__(256) int32_t g_noalloc_sums[kNoAllocSumElements];
static __device__ __align__(256) int g_noalloc_status[64];

struct NoAllocDevice {
    std::atomic<bool> ready{false};
    int32_t* sums = nullptr;
    int* status = nullptr;
    int sm_count = 0;
};

NoAllocDevice g_noalloc[64];
std::mutex g_noalloc_setup;

// The device addresses of the arrays for the current device, looked up on the first call on that device (host code
// may not use the symbols as addresses: they name host-side stand-ins). Host threads making their first call on one
// device at once are serialised by g_noalloc_setup; the fields are published by the release store of `ready`.
const NoAllocDevice& noalloc_device() {
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= 64)
        unsupported(kGemm, "device ordinal out of range for the allocation-free entry point", "Device", "< 64",
                    std::to_string(dev));
    NoAllocDevice& d = g_noalloc[dev];
    if (d.ready.load(std::memory_order_acquire)) return d;
    std::lock_guard<std::mutex> lock(g_noalloc_setup);
    if (!d.ready.load(std::memory_order_relaxed)) {
        void* sums = nullptr;
        void* status = nullptr;
        int sms = 0;
        check_cuda(cudaGetSymbolAddress(&sums, g_noalloc_sums), "cudaGetSymbolAddress");
        check_cuda(cudaGetSymbolAddress(&status, g_noalloc_status), "cudaGetSymbolAddress");
        check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
        d.sums = static_cast<int32_t*>(sums);
        d.status = static_cast<int*>(status);
        d.sm_count = sms;
        d.ready.store(true, std::memory_order_release);
    }
    return d;
}

}  // namespace

extern "C" {

OG_API og_status og_int8_gemm_int32_noalloc(void* stream, const og_int8_gemm_problem* p, const og_buffer* a,
                                            const og_buffer* b, const og_buffer* c, const og_operand* za,
                                            const og_operand* zb, const og_operand* bias) {
    return guard([&] {
        const Prepared pr = check_int32(p, a, b, c, za, zb, bias);
        if (!pr.ok) return;
        const NoAllocDevice& d = noalloc_device();
        og::GemmLaunch L = {};
        L.a = static_cast<const uint8_t*>(a->ptr) + p->offset_a;
        L.b = static_cast<const uint8_t*>(b->ptr) + p->offset_b;
        L.m = p->m;
        L.n = p->n;
        L.k = p->k;
        L.batch = p->batch;
        L.trans_b = p->transpose_b != 0;
        L.lda = pr.lda;
        L.ldb = pr.ldb;
        L.stride_a = p->stride_a;
        L.stride_b = p->stride_b;
        L.a_signed = a->type == OG_S8;
        L.b_signed = b->type == OG_S8;
        L.num_sms = d.sm_count;
        L.error_flag = d.status;
        L.tile = 0;
        og::Epilogue& e = L.epi;
        e.out_kind = og::OUT_I32;
        e.c = static_cast<int32_t*>(c->ptr) + p->offset_c;
        e.ldc = p->n;
        e.batch_stride_c = static_cast<int64_t>(p->m) * p->n;
        e.m = p->m;
        e.n = p->n;
        e.k = p->k;
        e.za = operand_ptr(za);
        e.za_vector = za ? za->is_vector : 0;
        e.za_signed = a->type == OG_S8;
        e.zb = operand_ptr(zb);
        e.zb_vector = zb ? zb->is_vector : 0;
        e.zb_signed = b->type == OG_S8;
        e.int_bias = reinterpret_cast<const int32_t*>(operand_ptr(bias));
        e.vec_ok = ((reinterpret_cast<uintptr_t>(e.c) & 15) == 0) && ((static_cast<int64_t>(p->n) * 4) % 16 == 0);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const bool tc = og::tc_eligible(L) && static_cast<int64_t>(L.m) * L.n * L.k >= (int64_t(1) << 16);
        if (!tc) {
            check_cuda(og::launch_gemm_simt(L, s), "og_int8_gemm_int32_noalloc");
            return;
        }
        const int ba = (L.batch > 1 && L.stride_a != 0) ? L.batch : 1;
        const int bb = (L.batch > 1 && L.stride_b != 0) ? L.batch : 1;
        const int64_t rows = e.zb != nullptr ? int64_t(ba) * L.m : 0;
        const int64_t cols = e.za != nullptr ? int64_t(bb) * L.n : 0;
        if (rows + cols > kNoAllocSumElements)
            unsupported(kGemm,
                        "og_int8_gemm_int32_noalloc keeps the byte sums of the zero-point correction in a fixed array "
                        "of " + std::to_string(kNoAllocSumElements) + " int32; this product needs " +
                            std::to_string(rows + cols) + " (use og_int8_gemm_encode_int32, which allocates)",
                        "NoAllocScratch", "at most " + std::to_string(kNoAllocSumElements) + " byte sums",
                        std::to_string(rows + cols) + " byte sums");
        if (rows + cols > 0) {
            e.row_sum_a = rows ? d.sums : nullptr;
            e.row_sum_a_stride = ba > 1 ? L.m : 0;
            e.col_sum_b = cols ? d.sums + rows : nullptr;
            e.col_sum_b_stride = bb > 1 ? L.n : 0;
            e.sum_splits = 1;  // launch_byte_sums writes whole sums
            e.row_sum_split_stride = rows;
            e.col_sum_split_stride = cols;
            check_cuda(og::launch_byte_sums(L, const_cast<int32_t*>(e.row_sum_a), const_cast<int32_t*>(e.col_sum_b), s),
                       "og_int8_gemm_int32_noalloc");
        }
        check_cuda(og::launch_gemm_tc(L, s), "og_int8_gemm_int32_noalloc");
    });
}

OG_API og_status og_int8_gemm_noalloc_status(void* stream) {
    return guard([&] {
        const NoAllocDevice& d = noalloc_device();
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        int word = 0;  // pageable host memory: the copy lands before cudaStreamSynchronize returns
        check_cuda(cudaMemcpyAsync(&word, d.status, sizeof(int), cudaMemcpyDeviceToHost, s), "status readback");
        check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        if (word != 0) {
            check_cuda(cudaMemsetAsync(d.status, 0, sizeof(int), s), "status reset");
            check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
            throw OgError{OG_ERROR_COMMAND_FAILED, kGemm, "",
                          "a kernel of an allocation-free product gave up waiting on its own pipeline (watchdog) and "
                          "skipped its work",
                          "Watchdog", "", ""};
        }
    });
}

OG_API og_status og_int8_gemm_noalloc_watchdog_selftest(void* stream, uint32_t limit_us) {
    return guard([&] {
        if (limit_us < 1 || limit_us > 2000000)
            throw OgError{OG_ERROR_ARGUMENT_RANGE, kGemm, "limitMicroseconds",
                          "the self-test wait limit is 1 .. 2000000 microseconds", "", "", ""};
        const NoAllocDevice& d = noalloc_device();
        og::watchdog_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(d.status,
                                                                                     uint64_t(limit_us) * 1000);
        check_cuda(cudaGetLastError(), "watchdog self-test launch");
    });
}

}  // extern "C"
