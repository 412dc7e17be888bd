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
//
// The unfolding (pack) kernels, by geometry: one-dimensional rows with width stride 1 or 2 (conv_pack_row_kernel: a
// warp per input row, register windows of aligned words), other planes that fit shared memory (conv_pack_plane_kernel:
// the plane staged and re-laid as phase rows, each output row then a contiguous slice), and the rest
// (conv_pack_kernel: gathers from global memory).
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
    uint32_t cin_g_magic, groups_magic;  // the same for n / cin_g and n / groups (the plane kernel's block index)
    int32_t cin_g_shift, groups_shift;
};

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

constexpr int64_t PLANE_SMEM_MAX = 160 * 1024;  // the plane kernel runs when its shared memory fits this

// Plane kernel: groups of TPP threads (a CTA holds PACK_THREADS / TPP of them, each with its own shared memory)
// walk input planes (image, group, channel c) in grid-stride order. A group stages its plane in shared memory (4-byte
// cp.async when every plane starts on a 4-byte boundary), re-lays it as phase rows (below), starts staging its next
// plane and meanwhile writes the KH * KW rows of the column matrix that the current plane feeds (rows c * KH * KW ..). Small planes get small groups, so the per-plane
// bookkeeping is not repeated by threads that have little else to do. A group first re-lays its plane as phase rows:
// for input row iy and phase r < SW, E[iy][r][j] = x[iy][j * SW + r - PW], the zero point where that column lies in
// the padding. Tap (kh, kw) of output (oy, ox) then reads E[oy * SH + kh * DH - PH][t % SW][ox + t / SW] with
// t = kw * DW: one output row is a contiguous slice of one phase row, copied 16 bytes per thread with two aligned
// 16-byte shared loads and funnel shifts, consecutive threads writing consecutive 16 bytes of the matrix row. Chunks
// that cross an output row, reach past OH * OW or lie in vertical padding go byte by byte.
struct PlaneLayout {
    int32_t hw;       // bytes of one input plane
    int32_t raw_pad;  // bytes of the staging buffer (hw rounded up to 16, plus 16)
    int32_t e_len;    // L: bytes of one phase row (a multiple of 16, covering every slice plus 32 bytes)
    int32_t group_bytes;  // shared memory of one group: the staging buffer and H * SW phase rows
    uint32_t sw_magic;    // t / SW by div_magic
    int32_t sw_shift;
    bool async;       // every plane starts 4-byte aligned and spans whole words
};

template <int TPP>
__device__ __forceinline__ void group_sync(int32_t group) {
    if constexpr (TPP == 32)
        __syncwarp();
    else
        asm volatile("bar.sync %0, %1;" ::"r"(group + 1), "r"(TPP) : "memory");
}

template <int TPP>
__device__ __forceinline__ void stage_plane(const PackArgs& a, const PlaneLayout& pl, int32_t plane, int32_t lane,
                                            uint8_t* dst) {
    const int32_t ig = div_magic(plane, a.cin_g_magic, a.cin_g_shift);
    const int32_t c = plane - ig * a.cin_g;
    const int32_t img = div_magic(ig, a.groups_magic, a.groups_shift);
    const int32_t g = ig - img * a.groups;
    const uint8_t* src = a.x + (static_cast<int64_t>(img) * a.cin + g * a.cin_g + c) * static_cast<int64_t>(pl.hw);
    if (pl.async) {
        const int32_t words = pl.hw >> 2;
        for (int32_t i = lane; i < words; i += TPP) cp_async4(dst + 4 * i, src + 4 * i);
    } else {
        for (int32_t i = lane; i < pl.hw; i += TPP) dst[i] = __ldg(src + i);
    }
}

// The 16 bytes of E starting at byte s (any alignment; E + s + 31 rounded down to 16 lies inside E).
__device__ __forceinline__ uint4 slice16(const uint8_t* __restrict__ e, int32_t s) {
    const uint4 v0 = *reinterpret_cast<const uint4*>(e + (s & ~15));
    const uint4 v1 = *reinterpret_cast<const uint4*>(e + (s & ~15) + 16);
    const uint32_t sh = 8 * (s & 3);
    uint32_t w0, w1, w2, w3, w4;
    switch ((s >> 2) & 3) {
        case 0: w0 = v0.x; w1 = v0.y; w2 = v0.z; w3 = v0.w; w4 = v1.x; break;
        case 1: w0 = v0.y; w1 = v0.z; w2 = v0.w; w3 = v1.x; w4 = v1.y; break;
        case 2: w0 = v0.z; w1 = v0.w; w2 = v1.x; w3 = v1.y; w4 = v1.z; break;
        default: w0 = v0.w; w1 = v1.x; w2 = v1.y; w3 = v1.z; w4 = v1.w; break;
    }
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}

// Four bytes of phase row r at j: x[iy][s + q * SW] for q < 4 with s = j * SW + r - PW, from the staged row `rrow`
// (padded by 16 readable bytes past the plane); word loads and byte permutes when all four lie inside the row.
template <int SW>
__device__ __forceinline__ uint32_t phase_word(const uint8_t* __restrict__ raw, int32_t row0, int32_t s, int32_t w,
                                               int32_t sw, uint32_t pad) {
    if (s >= 0 && s + 3 * sw < w) {
        const int32_t b = row0 + s;
        if constexpr (SW == 1) {
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(raw + (b & ~3));
            return __funnelshift_r(wp[0], wp[1], 8 * (b & 3));
        } else if constexpr (SW == 2) {
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(raw + (b & ~3));
            const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2];
            return __byte_perm(__funnelshift_r(w0, w1, 8 * (b & 3)), __funnelshift_r(w1, w2, 8 * (b & 3)), 0x6420);
        } else {
            return __byte_perm(__byte_perm(raw[b], raw[b + sw], 0x0040), __byte_perm(raw[b + 2 * sw], raw[b + 3 * sw], 0x0040),
                               0x5410);
        }
    }
    uint32_t v[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int32_t cq = s + q * sw;
        v[q] = static_cast<uint32_t>(cq) < static_cast<uint32_t>(w) ? raw[row0 + cq] : pad;
    }
    return __byte_perm(__byte_perm(v[0], v[1], 0x0040), __byte_perm(v[2], v[3], 0x0040), 0x5410);
}

template <int TPP, int SW>
__global__ void __launch_bounds__(PACK_THREADS) conv_pack_plane_kernel(const PackArgs a, int32_t planes,
                                                                       PlaneLayout pl) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int32_t GROUPS = PACK_THREADS / TPP;
    const int32_t group = static_cast<int32_t>(threadIdx.x) / TPP;
    const int32_t lane = static_cast<int32_t>(threadIdx.x) % TPP;
    uint8_t* const raw = smem + group * pl.group_bytes;  // the staged plane
    uint8_t* const e = raw + pl.raw_pad;                  // its phase rows, H * SW of them
    const uint32_t pad = a.zp != nullptr ? __ldg(a.zp) : 0u;
    const int32_t ncols = a.oh * a.ow;
    const int32_t taps = a.kh * a.kw;
    const int32_t chunks = a.ld >> 4;
    const int32_t stride = static_cast<int32_t>(gridDim.x) * GROUPS;
    const int32_t sw = SW != 0 ? SW : a.sw;
    int32_t p = static_cast<int32_t>(blockIdx.x) * GROUPS + group;
    if (p < planes) stage_plane<TPP>(a, pl, p, lane, raw);
    for (; p < planes; p += stride) {
        cp_async_wait_all();
        group_sync<TPP>(group);  // plane p is staged, and the group is done reading E
        // E, four bytes per thread and step.
        for (int32_t iy = 0; iy < a.h; iy++) {
            for (int32_t r = 0; r < sw; r++) {
                uint32_t* erow = reinterpret_cast<uint32_t*>(e + (iy * sw + r) * pl.e_len);
                for (int32_t j = 4 * lane; j < pl.e_len; j += 4 * TPP)
                    erow[j >> 2] = phase_word<SW>(raw, iy * a.w, j * sw + r - a.pw, a.w, sw, pad);
            }
        }
        group_sync<TPP>(group);  // E is complete and the staged plane is free: bring in the next one meanwhile
        const int32_t next = p + stride;
        if (next < planes) stage_plane<TPP>(a, pl, next, lane, raw);
        const int32_t ig = div_magic(p, a.cin_g_magic, a.cin_g_shift);
        const int32_t c = p - ig * a.cin_g;
        uint8_t* row_dst = a.cols + (static_cast<int64_t>(ig) * a.rows + static_cast<int64_t>(c) * taps) * a.ld;
        for (int32_t kh = 0; kh < a.kh; kh++) {
            const int32_t dy = kh * a.dh - a.ph;
            for (int32_t kw = 0; kw < a.kw; kw++, row_dst += a.ld) {
                const int32_t t = kw * a.dw;
                const int32_t q = div_magic(t, pl.sw_magic, pl.sw_shift);
                const int32_t rr = t - q * sw;
                for (int32_t u = lane; u < chunks; u += TPP) {
                    const int32_t col0 = u * 16;
                    const int32_t oy = div_magic(col0, a.ow_magic, a.ow_shift);
                    int32_t ox = col0 - oy * a.ow;
                    int32_t iy = oy * a.sh + dy;
                    uint4 out;
                    if (col0 + 16 <= ncols && ox + 16 <= a.ow && static_cast<uint32_t>(iy) < static_cast<uint32_t>(a.h)) {
                        out = slice16(e, (iy * sw + rr) * pl.e_len + ox + q);
                    } else {
                        uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int k = 0; k < 16; k++) {
                            uint32_t v = pad;
                            if (col0 + k < ncols && static_cast<uint32_t>(iy) < static_cast<uint32_t>(a.h))
                                v = e[(iy * sw + rr) * pl.e_len + ox + q];
                            w[k >> 2] |= v << (8 * (k & 3));
                            if (++ox == a.ow) {
                                ox = 0;
                                iy += a.sh;
                            }
                        }
                        out = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                    *reinterpret_cast<uint4*>(row_dst + col0) = out;
                }
            }
        }
    }
}

// One-dimensional convolutions (H = KH = 1) with width stride SW of 1 or 2 and taps spanning at most 8 input columns
// ((KW - 1) * DW <= 8): one warp per input row, each lane writing output words (four columns) of the row's KW matrix
// rows. For a word at ox0, every tap reads inside the input window [SW * ox0 - PW, SW * ox0 + 3 * SW + (KW - 1) * DW
// - PW]; the lane loads that window once as NW aligned words and forms each tap's word with funnel shifts (and, at
// stride 2, a byte permute picking every other byte). Words whose window leaves the row, or that reach past OW, go
// byte by byte with the padding rules. Two or four words per lane are in flight at once.
template <int SW>
struct RowWindow {
    static constexpr int NW = SW == 1 ? 4 : 5;  // words: an offset below 4 plus at most 8 + 3 * SW + 1 bytes
};

template <int SW, int I>
__device__ __forceinline__ uint32_t tap_word_at(const uint32_t (&w)[RowWindow<SW>::NW], uint32_t sh) {
    if constexpr (SW == 1) {
        return __funnelshift_r(w[I], w[I + 1], sh);
    } else {
        return __byte_perm(__funnelshift_r(w[I], w[I + 1], sh), __funnelshift_r(w[I + 1], w[I + 2], sh), 0x6420);
    }
}

// The tap word whose first byte is byte S of the window (S <= 11).
template <int SW>
__device__ __forceinline__ uint32_t tap_word(const uint32_t (&w)[RowWindow<SW>::NW], int32_t s) {
    const uint32_t sh = 8u * static_cast<uint32_t>(s & 3);
    switch (s >> 2) {
        case 0: return tap_word_at<SW, 0>(w, sh);
        case 1: return tap_word_at<SW, 1>(w, sh);
        default: return tap_word_at<SW, 2>(w, sh);
    }
}

// The KW tap words of one output word from its window, every position and shift a constant: taps of unit
// dilation, window offset O (KW > 0 only).
template <int SW, int O, int KW, int K = 0>
struct RowTaps {
    __device__ static __forceinline__ void store(const uint32_t (&w)[RowWindow<SW>::NW], uint8_t* dst, int32_t ld) {
        if constexpr (K < KW) {
            constexpr int S = K + O;
            *reinterpret_cast<uint32_t*>(dst) = tap_word_at<SW, (S >> 2)>(w, 8u * (S & 3));
            RowTaps<SW, O, KW, K + 1>::store(w, dst + ld, ld);
        }
    }
};

// One input row's output words. KW = 0: any tap count and dilation (tap positions found at run time); KW > 0: that
// many taps of unit dilation with the window offset O fixed.
template <bool SMEM>
__device__ __forceinline__ uint32_t row_word(const uint32_t* p) {
    if constexpr (SMEM)
        return *p;
    else
        return __ldg(p);
}
template <bool SMEM>
__device__ __forceinline__ uint32_t row_byte(const uint8_t* p) {
    if constexpr (SMEM)
        return *p;
    else
        return __ldg(p);
}

// `row` is the input row in global memory, or (SMEM) its copy in shared memory at the same offset modulo 8.
template <int SW, int KW, int O, bool SMEM = false>
__device__ __forceinline__ void row_words(const PackArgs& a, const uint8_t* row, uint8_t* dst0, int32_t o,
                                          int32_t lane, uint32_t pad) {
    constexpr int NW = RowWindow<SW>::NW;
    constexpr int U = KW > 0 ? 2 : 4;  // output words per lane in flight
    const int32_t words = a.ld >> 2;
    for (int32_t t0 = lane; t0 < words; t0 += 32 * U) {
        uint32_t win[U][NW];
        bool fast[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int32_t ox0 = 4 * (t0 + 32 * u);
            const int32_t lo = SW * ox0 - a.pw - o;  // first byte of the window's first word
            fast[u] = t0 + 32 * u < words && ox0 + 4 <= a.ow && lo >= 0 && lo + 4 * NW <= a.w;
            if (fast[u]) {
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(row + lo);
#pragma unroll
                for (int k = 0; k < NW; k++) win[u][k] = row_word<SMEM>(wp + k);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int32_t t = t0 + 32 * u;
            if (t >= words) break;
            const int32_t ox0 = 4 * t;
            uint8_t* dst = dst0 + ox0;
            if constexpr (KW > 0) {
                if (fast[u]) {
                    RowTaps<SW, O, KW>::store(win[u], dst, a.ld);
                    continue;
                }
            }
            for (int32_t kw = 0; kw < a.kw; kw++, dst += a.ld) {
                uint32_t word;
                if (KW == 0 && fast[u]) {
                    word = tap_word<SW>(win[u], kw * a.dw + o);
                } else {
                    word = 0;
                    const int32_t d = kw * a.dw - a.pw;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int32_t ix = SW * (ox0 + e) + d;
                        uint32_t v = pad;
                        if (ox0 + e < a.ow && static_cast<uint32_t>(ix) < static_cast<uint32_t>(a.w))
                            v = row_byte<SMEM>(row + ix);
                        word |= v << (8 * e);
                    }
                }
                *reinterpret_cast<uint32_t*>(dst) = word;
            }
        }
    }
}

template <int SW, int KW>
__global__ void __launch_bounds__(PACK_THREADS, 4) conv_pack_row_kernel(const PackArgs a, int32_t planes) {
    pdl_trigger();
    pdl_wait();
    const int32_t lane = static_cast<int32_t>(threadIdx.x) & 31;
    const int32_t warps = static_cast<int32_t>(gridDim.x) * (PACK_THREADS / 32);
    const uint32_t pad = a.zp != nullptr ? __ldg(a.zp) : 0u;
    for (int32_t plane = static_cast<int32_t>((blockIdx.x * PACK_THREADS + threadIdx.x) >> 5); plane < planes;
         plane += warps) {
        const int32_t ig = div_magic(plane, a.cin_g_magic, a.cin_g_shift);
        const int32_t c = plane - ig * a.cin_g;
        const int32_t img = div_magic(ig, a.groups_magic, a.groups_shift);
        const int32_t g = ig - img * a.groups;
        const uint8_t* row = a.x + (static_cast<int64_t>(img) * a.cin + g * a.cin_g + c) * static_cast<int64_t>(a.w);
        uint8_t* dst0 = a.cols + (static_cast<int64_t>(ig) * a.rows + static_cast<int64_t>(c) * a.kw) * a.ld;
        // Byte offset of the window's first byte within its aligned word (the same for every word of the row).
        const int32_t o = static_cast<int32_t>((reinterpret_cast<uintptr_t>(row) - static_cast<uintptr_t>(a.pw)) & 3);
        if constexpr (KW == 0) {
            row_words<SW, 0, 0>(a, row, dst0, o, lane, pad);
        } else {
            switch (o) {
                case 0: row_words<SW, KW, 0>(a, row, dst0, o, lane, pad); break;
                case 1: row_words<SW, KW, 1>(a, row, dst0, o, lane, pad); break;
                case 2: row_words<SW, KW, 2>(a, row, dst0, o, lane, pad); break;
                default: row_words<SW, KW, 3>(a, row, dst0, o, lane, pad); break;
            }
        }
    }
}

// The row kernel with each warp's rows staged in shared memory: while a warp packs one row from its copy, the next
// row of its grid-stride sequence is on its way (8-byte cp.async; the bytes before the row's first 8-byte boundary
// and after its last one by plain loads), so a warp keeps a whole row in flight instead of a few words per lane.
// The copy keeps the row's offset modulo 8, so the word windows are the row kernel's.
template <int SW, int KW>
__global__ void __launch_bounds__(PACK_THREADS, 2) conv_pack_row_staged_kernel(const PackArgs a, int32_t planes,
                                                                              int32_t cap) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t row_s[];
    const int32_t lane = static_cast<int32_t>(threadIdx.x) & 31;
    uint8_t* const bufs = row_s + (threadIdx.x >> 5) * 2 * cap;  // this warp's two row buffers
    const int32_t warps = static_cast<int32_t>(gridDim.x) * (PACK_THREADS / 32);
    const uint32_t pad = a.zp != nullptr ? __ldg(a.zp) : 0u;
    auto plane_row = [&](int32_t plane, int32_t& ig, int32_t& c) {
        ig = div_magic(plane, a.cin_g_magic, a.cin_g_shift);
        c = plane - ig * a.cin_g;
        const int32_t img = div_magic(ig, a.groups_magic, a.groups_shift);
        const int32_t g = ig - img * a.groups;
        return a.x + (static_cast<int64_t>(img) * a.cin + g * a.cin_g + c) * static_cast<int64_t>(a.w);
    };
    auto stage = [&](const uint8_t* row, uint8_t* buf) {
        uint8_t* dst = buf + (reinterpret_cast<uintptr_t>(row) & 7);
        int32_t head = static_cast<int32_t>((8 - (reinterpret_cast<uintptr_t>(row) & 7)) & 7);
        if (head > a.w) head = a.w;
        const int32_t chunks = (a.w - head) >> 3;
        for (int32_t i = lane; i < head; i += 32) dst[i] = __ldg(row + i);
        for (int32_t i = lane; i < chunks; i += 32) cp_async8(dst + head + 8 * i, row + head + 8 * i);
        for (int32_t i = head + 8 * chunks + lane; i < a.w; i += 32) dst[i] = __ldg(row + i);
        cp_async_commit();
    };
    int32_t plane = static_cast<int32_t>((blockIdx.x * PACK_THREADS + threadIdx.x) >> 5);
    int32_t it = 0, ig, c;
    if (plane < planes) stage(plane_row(plane, ig, c), bufs);
    for (; plane < planes; plane += warps, it++) {
        const uint8_t* row = plane_row(plane, ig, c);
        const int32_t next = plane + warps;
        if (next < planes) {
            int32_t ig2, c2;
            stage(plane_row(next, ig2, c2), bufs + ((it + 1) & 1) * cap);
        } else {
            cp_async_commit();  // an empty group keeps one group per step
        }
        cp_async_wait_group<1>();  // this row's copies are done
        __syncwarp();
        const uint8_t* srow = bufs + (it & 1) * cap + (reinterpret_cast<uintptr_t>(row) & 7);
        uint8_t* dst0 = a.cols + (static_cast<int64_t>(ig) * a.rows + static_cast<int64_t>(c) * a.kw) * a.ld;
        const int32_t o = static_cast<int32_t>((reinterpret_cast<uintptr_t>(row) - static_cast<uintptr_t>(a.pw)) & 3);
        if constexpr (KW == 0) {
            row_words<SW, 0, 0, true>(a, srow, dst0, o, lane, pad);
        } else {
            switch (o) {
                case 0: row_words<SW, KW, 0, true>(a, srow, dst0, o, lane, pad); break;
                case 1: row_words<SW, KW, 1, true>(a, srow, dst0, o, lane, pad); break;
                case 2: row_words<SW, KW, 2, true>(a, srow, dst0, o, lane, pad); break;
                default: row_words<SW, KW, 3, true>(a, srow, dst0, o, lane, pad); break;
            }
        }
        __syncwarp();  // the warp is done with this buffer before it is refilled
    }
    cp_async_wait_all();
}

static cudaError_t launch_conv_pack(const PackArgs& a, int64_t planes, int num_sms, cudaStream_t s) {
    const bool wide = a.ld % 16 == 0 && (reinterpret_cast<uintptr_t>(a.cols) & 15) == 0;
    const int64_t hw = static_cast<int64_t>(a.h) * a.w;
    // Phase rows: the longest slice is OW + (KW - 1) * DW / SW bytes; 32 more for the aligned 16-byte loads.
    const int64_t e_len = ((static_cast<int64_t>(a.ow) + (static_cast<int64_t>(a.kw) - 1) * a.dw / a.sw + 15) & ~15) + 32;
    const int64_t raw_pad = ((hw + 15) & ~15) + 16;  // 16 readable bytes past the plane for the word gathers
    const int64_t smem = raw_pad + static_cast<int64_t>(a.h) * a.sw * e_len;
    if (a.h == 1 && a.kh == 1 && a.oh == 1 && (a.sw == 1 || a.sw == 2) &&
        (static_cast<int64_t>(a.kw) - 1) * a.dw <= 8 && a.pw <= 8 && planes <= 0x7FFF0000) {
        const int64_t blocks = (planes + PACK_THREADS / 32 - 1) / (PACK_THREADS / 32);
        const int64_t cap = 8 * static_cast<int64_t>(num_sms);
        const unsigned grid = static_cast<unsigned>(blocks < cap ? blocks : cap);
        const int32_t np = static_cast<int32_t>(planes);
        // Rows up to ~6 KB are staged in shared memory (two buffers per warp, at least two CTAs per SM).
        const int64_t row_cap = ((static_cast<int64_t>(a.w) + 8 + 15) & ~int64_t(15));
        const int64_t smem = 2 * row_cap * (PACK_THREADS / 32);
        if (smem <= 100 * 1024) {
            int per_sm = static_cast<int>((200 * 1024) / smem);
            per_sm = per_sm < 1 ? 1 : (per_sm > 2 ? 2 : per_sm);  // its registers allow two CTAs per SM
            const int64_t resident = static_cast<int64_t>(per_sm) * num_sms;
            const unsigned sgrid = static_cast<unsigned>(blocks < resident ? blocks : resident);
            const int32_t c32 = static_cast<int32_t>(row_cap);
            const size_t bytes = static_cast<size_t>(smem);
            auto go = [&](auto kernel) -> cudaError_t {
                if (bytes > 48 * 1024) {
                    const cudaError_t e =
                        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
                    if (e != cudaSuccess) return e;
                }
                return launch_pdl(kernel, dim3(sgrid), dim3(PACK_THREADS), bytes, s, a, np, c32);
            };
            if (a.kw == 3 && a.dw == 1)
                return a.sw == 1 ? go(conv_pack_row_staged_kernel<1, 3>) : go(conv_pack_row_staged_kernel<2, 3>);
            return a.sw == 1 ? go(conv_pack_row_staged_kernel<1, 0>) : go(conv_pack_row_staged_kernel<2, 0>);
        }
        if (a.kw == 3 && a.dw == 1)  // the common three-tap kernel: every tap position a constant
            return a.sw == 1 ? launch_pdl(conv_pack_row_kernel<1, 3>, dim3(grid), dim3(PACK_THREADS), 0, s, a, np)
                             : launch_pdl(conv_pack_row_kernel<2, 3>, dim3(grid), dim3(PACK_THREADS), 0, s, a, np);
        return a.sw == 1 ? launch_pdl(conv_pack_row_kernel<1, 0>, dim3(grid), dim3(PACK_THREADS), 0, s, a, np)
                         : launch_pdl(conv_pack_row_kernel<2, 0>, dim3(grid), dim3(PACK_THREADS), 0, s, a, np);
    }
    if (wide && smem <= PLANE_SMEM_MAX && planes <= 0x7FFF0000) {  // grid-stride plane indices stay below 2^31
        // Threads per plane: about one per 96 bytes of plane, a power of two from 32 to 256.
        int tpp = 32;
        while (tpp < PACK_THREADS && static_cast<int64_t>(tpp) * 96 < hw) tpp *= 2;
        const int groups = PACK_THREADS / tpp;
        PlaneLayout pl;
        pl.hw = static_cast<int32_t>(hw);
        pl.raw_pad = static_cast<int32_t>(raw_pad);
        pl.e_len = static_cast<int32_t>(e_len);
        pl.group_bytes = static_cast<int32_t>(smem);
        magic_for(static_cast<uint32_t>(a.sw), &pl.sw_magic, &pl.sw_shift);
        pl.async = ((reinterpret_cast<uintptr_t>(a.x) | static_cast<uintptr_t>(hw)) & 3) == 0;
        // The grid covers the planes once, or fills the SMs with as many CTAs as the shared memory allows.
        const int64_t cta_smem = smem * groups;
        if (cta_smem > 200 * 1024) tpp = PACK_THREADS;  // (only reached for planes above 24 KB: one group)
        const int64_t cta_bytes = tpp == PACK_THREADS ? smem : cta_smem;
        int per_sm = static_cast<int>((200 * 1024) / cta_bytes);
        per_sm = per_sm < 1 ? 1 : (per_sm > 8 ? 8 : per_sm);
        const int g_per_cta = PACK_THREADS / tpp;
        const int64_t need = (planes + g_per_cta - 1) / g_per_cta;
        const int64_t resident = static_cast<int64_t>(per_sm) * num_sms;
        const unsigned grid = static_cast<unsigned>(need < resident ? need : resident);
        const size_t bytes = static_cast<size_t>(cta_bytes);
        auto go = [&](auto kernel) -> cudaError_t {
            if (bytes > 48 * 1024) {
                const cudaError_t e =
                    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
                if (e != cudaSuccess) return e;
            }
            return launch_pdl(kernel, dim3(grid), dim3(PACK_THREADS), bytes, s, a, static_cast<int32_t>(planes), pl);
        };
        const int swc = a.sw == 1 ? 1 : (a.sw == 2 ? 2 : 0);
        switch (tpp * 4 + swc) {
            case 32 * 4 + 1: return go(conv_pack_plane_kernel<32, 1>);
            case 32 * 4 + 2: return go(conv_pack_plane_kernel<32, 2>);
            case 32 * 4: return go(conv_pack_plane_kernel<32, 0>);
            case 64 * 4 + 1: return go(conv_pack_plane_kernel<64, 1>);
            case 64 * 4 + 2: return go(conv_pack_plane_kernel<64, 2>);
            case 64 * 4: return go(conv_pack_plane_kernel<64, 0>);
            case 128 * 4 + 1: return go(conv_pack_plane_kernel<128, 1>);
            case 128 * 4 + 2: return go(conv_pack_plane_kernel<128, 2>);
            case 128 * 4: return go(conv_pack_plane_kernel<128, 0>);
            case 256 * 4 + 1: return go(conv_pack_plane_kernel<256, 1>);
            case 256 * 4 + 2: return go(conv_pack_plane_kernel<256, 2>);
            default: return go(conv_pack_plane_kernel<256, 0>);
        }
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
            og::magic_for(static_cast<uint32_t>(cin_g), &a.cin_g_magic, &a.cin_g_shift);
            og::magic_for(static_cast<uint32_t>(p.groups), &a.groups_magic, &a.groups_shift);
            const int64_t planes = images * p.groups * cin_g;
            const int sms = cv->device->sm_count;
            enc->ops.push_back([=](cudaStream_t s) { return og::launch_conv_pack(a, planes, sms, s); });
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
