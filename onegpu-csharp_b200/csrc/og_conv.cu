// ConvIntegerKernels (ConvIntegerKernels.cs:25-351): ONNX ConvInteger,
//   y[n, m, oh, ow] = sum over c, kh, kw of (x - xZeroPoint) * (w[m, c, kh, kw] - wZeroPoint[m])   (wrapping int32)
// lowered, as the reference lowers it, to the int8 product after Chellapilla et al. (2006): one pass unfolds the
// windows of every image and group into a byte matrix of K = InChannels / Groups * KernelHeight * KernelWidth rows
// and OH * OW columns (Shaders/ConvIntegerPack.hlsl:1-12), then Int8Gemm.EncodeInt32 multiplies the weights of the
// group (A: OutChannels / Groups x K, zero point per row = per output channel) by it (B: K x OH*OW, the zero point of
// x), writing y's [OutChannels / Groups, OH * OW] block of the image directly.
//
// Differences of layout, none of result:
//  * the column matrix's rows are padded to 16 bytes (the reference pads to 4), so that the product loads it with
//    TMA and runs on the tensor cores; when caller scratch is too small for that padding, the reference's 4-byte
//    padding is used (the product then takes its portable path for unaligned rows);
//  * weights whose rows do not start on 16-byte boundaries are copied once per call into a pitched buffer of the
//    instance (rows padded to 16 bytes) for the same reason;
//  * without caller scratch, the batch runs in chunks of at most 256 MiB of columns (the reference: 64 MiB).
// A padded position holds the zero point of x, so after the product subtracts that zero point it adds nothing.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "og_gemm.h"
#include "og_host.h"
#include "og_ptx.cuh"

namespace og {

constexpr int PACK_THREADS = 256;

struct PackArgs {
    const uint8_t* x;   // first element of the first image of the chunk
    uint8_t* cols;      // first byte of the chunk's column matrices
    const uint8_t* zp;  // zero point of x, or null (pad with 0)
    int64_t units;      // BYTES-wide units of the chunk to write
    int32_t units_per_row;
    int32_t rows;       // K
    int32_t groups, cin, cin_g, h, w, oh, ow, kh, kw, sh, sw, dh, dw, ph, pw;
    int32_t ld;         // bytes per matrix row
    uint32_t ow_magic;  // n / ow = (umulhi(ow_magic, n) + n) >> ow_shift for 0 <= n < 2^31
    int32_t ow_shift;
};

// n / d for 0 <= n < 2^31 by multiplication (Granlund and Montgomery, "Division by Invariant Integers using
// Multiplication", 1994): magic and shift from magic_for(d).
__device__ __forceinline__ int32_t div_magic(int32_t n, uint32_t magic, int32_t shift) {
    return static_cast<int32_t>((__umulhi(magic, static_cast<uint32_t>(n)) + static_cast<uint32_t>(n)) >> shift);
}

static void magic_for(uint32_t d, uint32_t* magic, int32_t* shift) {
    int32_t l = 0;
    while ((uint64_t(1) << l) < d) l++;  // ceil(log2 d)
    *magic = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
    *shift = l;
}

// Unit t covers BYTES consecutive columns of one matrix row: row (c * KH + kh) * KW + kw of matrix (image, group)
// holds x[image, g * CinG + c, oh * SH - PH + kh * DH, ow * SW - PW + kw * DW] at column oh * OW + ow, or the zero
// point where that position lies in the padding or the column lies past OH * OW (ConvIntegerPack.hlsl:55-89).
template <int BYTES>
__global__ void __launch_bounds__(PACK_THREADS) conv_pack_kernel(const PackArgs a) {
    pdl_trigger();
    pdl_wait();
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= a.units) return;
    const int64_t r = t / a.units_per_row;
    const int32_t col0 = static_cast<int32_t>(t - r * a.units_per_row) * BYTES;
    const int32_t k = static_cast<int32_t>(r % a.rows);
    const int64_t ig = r / a.rows;
    const int64_t img = ig / a.groups;
    const int32_t g = static_cast<int32_t>(ig - img * a.groups);
    const int32_t taps = a.kh * a.kw;
    const int32_t c = k / taps;
    const int32_t kk = k - c * taps;
    const int32_t kh = kk / a.kw;
    const int32_t kw = kk - kh * a.kw;
    const uint8_t* plane = a.x + ((img * a.cin + g * a.cin_g + c) * static_cast<int64_t>(a.h)) * a.w;
    const uint32_t pad = a.zp != nullptr ? __ldg(a.zp) : 0u;
    const int32_t ncols = a.oh * a.ow;
    int32_t oy = col0 / a.ow;
    int32_t ox = col0 - oy * a.ow;
    uint32_t word[BYTES / 4];
#pragma unroll
    for (int q = 0; q < BYTES / 4; q++) word[q] = 0;
#pragma unroll
    for (int e = 0; e < BYTES; e++) {
        uint32_t v = pad;
        if (col0 + e < ncols) {
            const int32_t iy = oy * a.sh + kh * a.dh - a.ph;
            const int32_t ix = ox * a.sw + kw * a.dw - a.pw;
            if (static_cast<uint32_t>(iy) < static_cast<uint32_t>(a.h) && static_cast<uint32_t>(ix) < static_cast<uint32_t>(a.w))
                v = __ldg(plane + static_cast<int64_t>(iy) * a.w + ix);
        }
        word[e >> 2] |= v << (8 * (e & 3));
        if (++ox == a.ow) {
            ox = 0;
            oy++;
        }
    }
    uint8_t* dst = a.cols + r * a.ld + col0;
    if constexpr (BYTES == 16)
        *reinterpret_cast<uint4*>(dst) = make_uint4(word[0], word[1], word[2], word[3]);
    else
        *reinterpret_cast<uint32_t*>(dst) = word[0];
}

constexpr int PLANE_SMEM_MAX = 48 * 1024;  // planes up to this size are staged in shared memory

// One CTA per input plane (image, group, channel c): the plane is read once, with coalesced loads, into shared
// memory; then the CTA writes the KH * KW rows of the column matrix that plane feeds (rows c * KH * KW ..), BYTES
// columns per thread and store, every byte gathered from shared memory.
template <int BYTES>
__global__ void __launch_bounds__(PACK_THREADS) conv_pack_plane_kernel(const PackArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ uint8_t plane_s[];
    const int64_t plane = blockIdx.x;  // (image * groups + g) * cin_g + c
    const int32_t c = static_cast<int32_t>(plane % a.cin_g);
    const int64_t ig = plane / a.cin_g;
    const int64_t img = ig / a.groups;
    const int32_t g = static_cast<int32_t>(ig - img * a.groups);
    const int32_t hw = a.h * a.w;
    const uint8_t* src = a.x + (img * a.cin + g * a.cin_g + c) * static_cast<int64_t>(hw);
    if ((reinterpret_cast<uintptr_t>(src) & 3) == 0) {
        const int32_t words = hw >> 2;
        for (int32_t i = threadIdx.x; i < words; i += PACK_THREADS)
            reinterpret_cast<uint32_t*>(plane_s)[i] = __ldg(reinterpret_cast<const uint32_t*>(src) + i);
        for (int32_t i = (words << 2) + threadIdx.x; i < hw; i += PACK_THREADS) plane_s[i] = __ldg(src + i);
    } else {
        for (int32_t i = threadIdx.x; i < hw; i += PACK_THREADS) plane_s[i] = __ldg(src + i);
    }
    __syncthreads();
    const uint32_t pad = a.zp != nullptr ? __ldg(a.zp) : 0u;
    const int32_t taps = a.kh * a.kw;
    const int32_t ncols = a.oh * a.ow;
    // A plane's items (taps x units of one matrix row) fit 32-bit arithmetic, which is far cheaper than 64-bit here.
    const int32_t upr = a.units_per_row;
    uint8_t* rows0 = a.cols + (ig * a.rows + static_cast<int64_t>(c) * taps) * a.ld;
    // Taps in the outer loop (uniform, no division per item); the output position of a unit's first column by one
    // multiply-high (div_magic). Output (oy, ox) reads input row oy * SH + dy, column ox * SW + dx.
    for (int32_t kk = 0; kk < taps; kk++) {
        const int32_t kh = kk / a.kw;
        const int32_t kw = kk - kh * a.kw;
        const int32_t dy = kh * a.dh - a.ph;
        const int32_t dx = kw * a.dw - a.pw;
        uint8_t* row_dst = rows0 + static_cast<int64_t>(kk) * a.ld;
        for (int32_t u = threadIdx.x; u < upr; u += PACK_THREADS) {
            const int32_t col0 = u * BYTES;
            int32_t oy = div_magic(col0, a.ow_magic, a.ow_shift);
            int32_t ox = col0 - oy * a.ow;
            int32_t iy = oy * a.sh + dy;
            int32_t ix = ox * a.sw + dx;
            uint32_t word[BYTES / 4];
#pragma unroll
            for (int q = 0; q < BYTES / 4; q++) word[q] = 0;
#pragma unroll
            for (int e = 0; e < BYTES; e++) {
                uint32_t v = pad;
                if (col0 + e < ncols && static_cast<uint32_t>(iy) < static_cast<uint32_t>(a.h) &&
                    static_cast<uint32_t>(ix) < static_cast<uint32_t>(a.w))
                    v = plane_s[iy * a.w + ix];
                word[e >> 2] |= v << (8 * (e & 3));
                ix += a.sw;
                if (++ox == a.ow) {
                    ox = 0;
                    ix = dx;
                    iy += a.sh;
                }
            }
            uint8_t* dst = row_dst + col0;
            if constexpr (BYTES == 16)
                *reinterpret_cast<uint4*>(dst) = make_uint4(word[0], word[1], word[2], word[3]);
            else
                *reinterpret_cast<uint32_t*>(dst) = word[0];
        }
    }
}

static cudaError_t launch_conv_pack(const PackArgs& a, int64_t planes, cudaStream_t s) {
    const bool wide = a.ld % 16 == 0 && (reinterpret_cast<uintptr_t>(a.cols) & 15) == 0;
    const int32_t hw = a.h * a.w;
    if (hw <= PLANE_SMEM_MAX && planes <= 0x7FFFFFFF) {
        const unsigned grid = static_cast<unsigned>(planes);
        const size_t smem = static_cast<size_t>((hw + 15) & ~15);
        // Four columns per thread: adjacent lanes gather from shared memory 4 * stride bytes apart (at most 2-way
        // bank conflicts at stride 2, none at stride 1), and each warp stores 128 contiguous bytes.
        PackArgs b = a;
        b.units_per_row = a.ld / 4;
        b.units = a.units * (a.ld / 4) / a.units_per_row;
        return launch_pdl(conv_pack_plane_kernel<4>, dim3(grid), dim3(PACK_THREADS), smem, s, b);
    }
    const unsigned blocks = static_cast<unsigned>((a.units + PACK_THREADS - 1) / PACK_THREADS);
    return wide ? launch_pdl(conv_pack_kernel<16>, dim3(blocks), dim3(PACK_THREADS), 0, s, a)
                : launch_pdl(conv_pack_kernel<4>, dim3(blocks), dim3(PACK_THREADS), 0, s, a);
}

}  // namespace og

// ---- host side ----------------------------------------------------------------------------------------------------

struct og_conv_integer {
    og_device* device = nullptr;
    og_int8_gemm* gemm = nullptr;
    std::vector<void*> buffers;  // own columns / packed weights; older ones live until destroy (recorded work names them)
    void* columns = nullptr;
    int64_t columns_bytes = 0;
    void* weights = nullptr;
    int64_t weights_bytes = 0;
};

namespace {

using namespace og_host;

const char* kConv = "ConvInteger";
constexpr int64_t kOwnColumnBytes = int64_t(256) << 20;

// Raises the error an inner C ABI call left (the product's checks name their own arguments).
void forward(og_status st) {
    if (st == OG_OK) return;
    og_error_info info = {};
    og_last_error(&info);
    throw OgError{st, info.operation, info.argument, info.message, info.capability, info.expected, info.actual};
}

// ConvKernels.CheckWindow (ConvKernels.cs:895-926).
void check_window(const char* axis, int32_t input, int32_t kernel, int32_t stride, int32_t dilation, int32_t pad_begin,
                  int32_t pad_end) {
    const std::string a(axis);
    if (input < 1) shape(kConv, a + " input", "extent " + std::to_string(input) + " must be at least 1");
    if (kernel < 1) shape(kConv, a + " kernel", "extent " + std::to_string(kernel) + " must be at least 1");
    if (stride < 1) shape(kConv, a + " stride", "stride " + std::to_string(stride) + " must be at least 1");
    if (dilation < 1) shape(kConv, a + " dilation", "dilation " + std::to_string(dilation) + " must be at least 1");
    if (pad_begin < 0 || pad_end < 0)
        shape(kConv, a + " padding",
              "padding " + std::to_string(pad_begin) + ", " + std::to_string(pad_end) + " must not be negative");
    if (int64_t(kernel) * dilation > kMaxElements || int64_t(pad_begin) + pad_end + input > kMaxElements)
        shape(kConv, a, "the window or padding is larger than the supported sizes");
}

// GpuWindow.OutputExtent without auto padding or ceil mode (ConvProblem.cs OutHeight / OutWidth).
int32_t out_extent(int32_t input, int32_t kernel, int32_t stride, int32_t dilation, int32_t pad_begin, int32_t pad_end) {
    if (input < 1 || kernel < 1 || stride < 1 || dilation < 1) return 0;
    const int64_t effective = int64_t(dilation) * (kernel - 1) + 1;
    const int64_t span = int64_t(input) + pad_begin + pad_end - effective;
    if (span < 0) return 0;
    const int64_t extent = span / stride + 1;
    return extent > kMaxElements ? 0 : static_cast<int32_t>(extent);
}

struct ConvGeometry {
    int32_t oh = 0, ow = 0;
    int64_t k = 0, ldb = 0;  // rows of one column matrix, the reference's row length (OH*OW rounded up to 4)
};

// ConvIntegerKernels.Geometry (ConvIntegerKernels.cs:302-323) with ConvKernels.CheckConv (ConvKernels.cs:928-956).
ConvGeometry geometry(const og_conv_problem* p) {
    if (p == nullptr) null_arg(kConv, "problem");
    ConvGeometry g;
    g.oh = out_extent(p->height, p->kernel_height, p->stride_height, p->dilation_height, p->pad_top, p->pad_bottom);
    g.ow = out_extent(p->width, p->kernel_width, p->stride_width, p->dilation_width, p->pad_left, p->pad_right);
    if (p->batch < 1) shape(kConv, "Batch", "batch " + std::to_string(p->batch) + " must be at least 1");
    if (p->in_channels < 1 || p->out_channels < 1)
        shape(kConv, p->in_channels < 1 ? "InChannels" : "OutChannels",
              "channel counts " + std::to_string(p->in_channels) + ", " + std::to_string(p->out_channels) +
                  " must be at least 1");
    if (p->groups < 1 || p->in_channels % p->groups != 0 || p->out_channels % p->groups != 0)
        shape(kConv, "Groups",
              std::to_string(p->groups) + " groups do not divide " + std::to_string(p->in_channels) + " input and " +
                  std::to_string(p->out_channels) + " output channels");
    check_window("height", p->height, p->kernel_height, p->stride_height, p->dilation_height, p->pad_top,
                 p->pad_bottom);
    check_window("width", p->width, p->kernel_width, p->stride_width, p->dilation_width, p->pad_left, p->pad_right);
    if (g.oh < 1)
        shape(kConv, "height",
              "the kernel (" + std::to_string(p->kernel_height) + " with dilation " +
                  std::to_string(p->dilation_height) + ") does not fit the padded input (" +
                  std::to_string(p->height) + " + " + std::to_string(p->pad_top) + " + " +
                  std::to_string(p->pad_bottom) + ")");
    if (g.ow < 1)
        shape(kConv, "width",
              "the kernel (" + std::to_string(p->kernel_width) + " with dilation " + std::to_string(p->dilation_width) +
                  ") does not fit the padded input (" + std::to_string(p->width) + " + " +
                  std::to_string(p->pad_left) + " + " + std::to_string(p->pad_right) + ")");
    g.k = int64_t(p->in_channels / p->groups) * p->kernel_height * p->kernel_width;
    g.ldb = (int64_t(g.oh) * g.ow + 3) / 4 * 4;
    const int64_t x_all = int64_t(p->batch) * p->in_channels * p->height * p->width;
    if (g.k > kMaxElements || g.ldb > kMaxElements || x_all > kMaxElements)
        shape(kConv, "shape", "the convolution is larger than the supported sizes");
    return g;
}

void require_int8(const og_buffer* b, const char* arg) {
    if (b->type != OG_U8 && b->type != OG_S8)
        shape(kConv, arg, std::string("element type ") + type_name(b->type) +
                              " is not supported; use byte (uint8) or sbyte (int8)");
}

struct ConvPlan {
    ConvGeometry g;
    int64_t n_cols = 0, x_image = 0, y_image = 0, per_image = 0;
};

// ConvIntegerKernels.Encode's checks in the reference's order (ConvIntegerKernels.cs:106-184).
ConvPlan check_conv(const og_conv_problem* p, const og_buffer* x, const og_buffer* w, const og_buffer* y,
                    const og_operand* xz, const og_operand* wz, const og_buffer* scratch, int32_t scratch_offset) {
    if (x == nullptr) null_arg(kConv, "x");
    if (w == nullptr) null_arg(kConv, "w");
    if (y == nullptr) null_arg(kConv, "y");
    require_int8(x, "x");
    require_int8(w, "w");
    ConvPlan c;
    c.g = geometry(p);
    c.n_cols = int64_t(c.g.oh) * c.g.ow;
    if (p->activation != 0) shape(kConv, "Activation", "an integer convolution has no fused activation");
    if (y->type != OG_I32)
        shape(kConv, "y", std::string("element type ") + type_name(y->type) + " is not supported; use int");
    c.x_image = int64_t(p->in_channels) * p->height * p->width;
    c.y_image = int64_t(p->out_channels) * c.n_cols;
    range(kConv, "x", x->length, p->offset_x, c.x_image * p->batch);
    range(kConv, "w", w->length, p->offset_w, int64_t(p->out_channels) * c.g.k);
    range(kConv, "y", y->length, p->offset_y, c.y_image * p->batch);
    if (p->offset_y < 0 || int64_t(p->offset_y) + c.y_image * p->batch > kMaxElements)
        shape(kConv, "y", "the result is larger than the supported sizes");
    if (xz != nullptr) {
        if (xz->buffer.ptr == nullptr) null_arg(kConv, "xZeroPoint");
        if (xz->buffer.type != x->type)
            shape(kConv, "xZeroPoint", std::string("element type ") + type_name(xz->buffer.type) +
                                           " differs from the type of x, " + type_name(x->type));
        range(kConv, "xZeroPoint", xz->buffer.length, xz->offset, 1);
        if (xz->is_vector) shape(kConv, "xZeroPoint", "the zero point of x is a single value");
    }
    if (wz != nullptr) {
        if (wz->buffer.ptr == nullptr) null_arg(kConv, "wZeroPoint");
        if (wz->buffer.type != w->type)
            shape(kConv, "wZeroPoint", std::string("element type ") + type_name(wz->buffer.type) +
                                           " differs from the type of w, " + type_name(w->type));
        range(kConv, "wZeroPoint", wz->buffer.length, wz->offset, wz->is_vector ? p->out_channels : 1);
    }
    c.per_image = int64_t(p->groups) * c.g.k * c.g.ldb;
    if (c.per_image > kMaxElements)
        shape(kConv, "InChannels",
              "the column matrix of one image needs " + std::to_string(c.per_image) +
                  " bytes, more than the supported sizes");
    if (scratch != nullptr) {
        if (scratch_offset < 0 || (scratch_offset & 3) != 0)
            shape(kConv, "scratchOffset",
                  "offset " + std::to_string(scratch_offset) + " must be a non-negative multiple of 4");
        if (int64_t(scratch_offset) + c.per_image > scratch->length)
            shape(kConv, "scratch",
                  "bytes " + std::to_string(scratch_offset) + ".." + std::to_string(scratch_offset + c.per_image) +
                      " (one image's columns) reach past the buffer of " + std::to_string(scratch->length));
        if (scratch->type != x->type)
            shape(kConv, "scratch", std::string("element type ") + type_name(scratch->type) +
                                        " differs from the type of x, " + type_name(x->type));
    }
    return c;
}

// A device buffer of the instance of at least `bytes`, grown geometrically; a replaced one stays alive until destroy.
void* own(og_conv_integer* cv, void*& slot, int64_t& have, int64_t bytes) {
    if (slot != nullptr && have >= bytes) return slot;
    int64_t want = std::max<int64_t>(bytes, 4096);
    if (slot != nullptr) want = std::max(want, have * 2);
    void* p = nullptr;
    check_cuda(cudaMalloc(&p, static_cast<size_t>(want)), "ConvInteger columns");
    cv->buffers.push_back(p);
    slot = p;
    have = want;
    return p;
}

og_int8_gemm_problem gemm_problem(int32_t m, int64_t n, int64_t k) {
    og_int8_gemm_problem gp = {};
    gp.m = m;
    gp.n = static_cast<int32_t>(n);
    gp.k = static_cast<int32_t>(k);
    gp.batch = 1;
    return gp;
}

}  // namespace

extern "C" {

OG_API og_status og_conv_integer_create(og_device* d, const og_int8_gemm_options* options, og_conv_integer** out) {
    return guard([&] {
        if (d == nullptr) null_arg(kConv, "device");
        if (out == nullptr) null_arg(kConv, "out");
        auto* cv = new og_conv_integer();
        cv->device = d;
        const og_status st = og_int8_gemm_create(d, options, &cv->gemm);
        if (st != OG_OK) {
            delete cv;
            forward(st);
        }
        *out = cv;
    });
}

OG_API og_status og_conv_integer_destroy(og_conv_integer* cv) {
    return guard([&] {
        if (cv == nullptr) return;
        use(cv->device);
        cudaStreamSynchronize(cv->device->stream);
        for (void* p : cv->buffers) cudaFree(p);
        og_int8_gemm_destroy(cv->gemm);
        delete cv;
    });
}

OG_API og_status og_conv_integer_variant(og_conv_integer* cv, char* buffer, uint64_t capacity) {
    return guard([&] {
        if (cv == nullptr) throw OgError{OG_ERROR_INVALID_HANDLE, kConv, "conv", "null handle", "", "", ""};
        forward(og_int8_gemm_variant(cv->gemm, buffer, capacity));
    });
}

OG_API og_status og_conv_integer_bind_groups_created(og_conv_integer* cv, int32_t* count) {
    return guard([&] {
        if (cv == nullptr) throw OgError{OG_ERROR_INVALID_HANDLE, kConv, "conv", "null handle", "", "", ""};
        if (count == nullptr) null_arg(kConv, "count");
        forward(og_int8_gemm_bind_groups_created(cv->gemm, count));
        *count += static_cast<int32_t>(cv->buffers.size());  // device buffers the instance allocated
    });
}

OG_API og_status og_conv_integer_scratch_bytes_per_image(const og_conv_problem* problem, int64_t* bytes) {
    return guard([&] {
        if (bytes == nullptr) null_arg(kConv, "bytes");
        const ConvGeometry g = geometry(problem);
        *bytes = int64_t(problem->groups) * g.k * g.ldb;
    });
}

OG_API og_status og_conv_integer_check(const og_conv_problem* problem, const og_buffer* x, const og_buffer* w,
                                       const og_buffer* y, const og_operand* x_zero_point,
                                       const og_operand* w_zero_point, const og_buffer* scratch,
                                       int32_t scratch_offset) {
    return guard([&] {
        if (problem == nullptr) null_arg(kConv, "problem");
        check_conv(problem, x, w, y, x_zero_point, w_zero_point, scratch, scratch_offset);
    });
}

OG_API og_status og_conv_integer_encode(og_conv_integer* cv, og_encoder* enc, const og_conv_problem* problem,
                                        const og_buffer* x, const og_buffer* w, const og_buffer* y,
                                        const og_operand* x_zero_point, const og_operand* w_zero_point,
                                        const og_buffer* scratch, int32_t scratch_offset) {
    return guard([&] {
        if (cv == nullptr) throw OgError{OG_ERROR_INVALID_HANDLE, kConv, "conv", "null handle", "", "", ""};
        if (enc == nullptr) null_arg(kConv, "encoder");
        if (problem == nullptr) null_arg(kConv, "problem");
        const og_conv_problem p = *problem;
        const ConvPlan c = check_conv(&p, x, w, y, x_zero_point, w_zero_point, scratch, scratch_offset);
        use(cv->device);
        const int32_t cin_g = p.in_channels / p.groups, cout_g = p.out_channels / p.groups;
        const int64_t k = c.g.k;

        // Column rows of 16 bytes where the scratch allows it (tensor-core loads), else the reference's 4.
        const int64_t ld16 = (c.n_cols + 15) / 16 * 16;
        const int64_t per16 = int64_t(p.groups) * k * ld16;
        int64_t ld, per_image, images_per_chunk;
        uint8_t* col_base;
        int64_t col_len;
        if (scratch != nullptr) {
            const int64_t room = scratch->length - scratch_offset;
            ld = room >= per16 ? ld16 : c.g.ldb;
            per_image = int64_t(p.groups) * k * ld;
            images_per_chunk = std::min<int64_t>(p.batch, room / per_image);
            col_base = static_cast<uint8_t*>(scratch->ptr) + scratch_offset;
            col_len = room;
        } else {
            ld = ld16;
            per_image = per16;
            images_per_chunk = std::max<int64_t>(1, std::min<int64_t>(p.batch, kOwnColumnBytes / per_image));
            col_len = images_per_chunk * per_image;
            col_base = static_cast<uint8_t*>(own(cv, cv->columns, cv->columns_bytes, col_len));
        }
        const og_buffer cols{col_base, col_len, x->type};

        // The weights as the product's A: w itself when its rows can be loaded by TMA, else a pitched copy.
        const uint8_t* w_first = static_cast<const uint8_t*>(w->ptr) + p.offset_w;
        og_buffer wa{const_cast<uint8_t*>(w_first), w->length - p.offset_w, w->type};
        int64_t lda = k;
        if ((k & 15) != 0 || (reinterpret_cast<uintptr_t>(w_first) & 15) != 0) {
            lda = (k + 15) / 16 * 16;
            const int64_t bytes = lda * p.out_channels;
            void* dst = own(cv, cv->weights, cv->weights_bytes, bytes);
            const int64_t rows = p.out_channels;
            enc->ops.push_back([=](cudaStream_t s) {
                return cudaMemcpy2DAsync(dst, static_cast<size_t>(lda), w_first, static_cast<size_t>(k),
                                         static_cast<size_t>(k), static_cast<size_t>(rows), cudaMemcpyDeviceToDevice,
                                         s);
            });
            wa = og_buffer{dst, bytes, w->type};
        }

        const uint8_t* xz_ptr = x_zero_point != nullptr
                                    ? static_cast<const uint8_t*>(x_zero_point->buffer.ptr) + x_zero_point->offset
                                    : nullptr;
        for (int64_t first = 0; first < p.batch; first += images_per_chunk) {
            const int64_t images = std::min<int64_t>(images_per_chunk, p.batch - first);
            og::PackArgs a{};
            a.x = static_cast<const uint8_t*>(x->ptr) + p.offset_x + first * c.x_image;
            a.cols = col_base;
            a.zp = xz_ptr;
            a.ld = static_cast<int32_t>(ld);
            const int bytes_per_unit = (ld % 16 == 0 && (reinterpret_cast<uintptr_t>(col_base) & 15) == 0) ? 16 : 4;
            a.units_per_row = static_cast<int32_t>(ld / bytes_per_unit);
            a.rows = static_cast<int32_t>(k);
            a.units = images * p.groups * k * a.units_per_row;
            a.groups = p.groups;
            a.cin = p.in_channels;
            a.cin_g = cin_g;
            a.h = p.height;
            a.w = p.width;
            a.oh = c.g.oh;
            a.ow = c.g.ow;
            a.kh = p.kernel_height;
            a.kw = p.kernel_width;
            a.sh = p.stride_height;
            a.sw = p.stride_width;
            a.dh = p.dilation_height;
            a.dw = p.dilation_width;
            a.ph = p.pad_top;
            a.pw = p.pad_left;
            og::magic_for(static_cast<uint32_t>(c.g.ow), &a.ow_magic, &a.ow_shift);
            const int64_t planes = images * p.groups * cin_g;
            enc->ops.push_back([=](cudaStream_t s) { return og::launch_conv_pack(a, planes, s); });
            enc->dispatches += 1;

            if (p.groups == 1) {
                og_int8_gemm_problem gp = gemm_problem(p.out_channels, c.n_cols, k);
                gp.batch = static_cast<int32_t>(images);
                gp.lda = static_cast<int32_t>(lda);
                gp.ldb = static_cast<int32_t>(ld);
                gp.offset_c = static_cast<int32_t>(p.offset_y + first * c.y_image);
                gp.stride_a = 0;
                gp.stride_b = static_cast<int32_t>(k * ld);
                forward(og_int8_gemm_encode_int32(cv->gemm, enc, &gp, &wa, &cols, y, w_zero_point, x_zero_point,
                                                  nullptr));
                continue;
            }
            for (int64_t img = 0; img < images; img++) {
                for (int32_t g = 0; g < p.groups; g++) {
                    og_int8_gemm_problem gp = gemm_problem(cout_g, c.n_cols, k);
                    gp.lda = static_cast<int32_t>(lda);
                    gp.ldb = static_cast<int32_t>(ld);
                    gp.offset_a = static_cast<int32_t>(int64_t(g) * cout_g * lda);
                    gp.offset_b = static_cast<int32_t>((img * p.groups + g) * k * ld);
                    gp.offset_c = static_cast<int32_t>(p.offset_y + (first + img) * c.y_image + int64_t(g) * cout_g * c.n_cols);
                    og_operand wzg;
                    const og_operand* wzp = w_zero_point;
                    if (w_zero_point != nullptr && w_zero_point->is_vector) {
                        wzg = *w_zero_point;
                        wzg.offset += g * cout_g;
                        wzp = &wzg;
                    }
                    forward(og_int8_gemm_encode_int32(cv->gemm, enc, &gp, &wa, &cols, y, wzp, x_zero_point, nullptr));
                }
            }
        }
    });
}

}  // extern "C"
