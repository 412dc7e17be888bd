// Multi-GPU plumbing of the C ABI: NCCL communicators over NVLink, used only to move sharded operands and results
// between the GPUs of one node (one process or thread per GPU). The product itself shards with no reduction, so
// there is no collective in its data path; these calls gather N-sharded results onto the device that needs them and
// replicate an operand that each rank uploaded one part of. The reference runs every device on its own with no
// cross-device traffic (MultiDeviceTests.cs:6-107), so nothing here has a counterpart there.
//
// NCCL is reached through dlopen("libnccl.so.2") at the first use, so the library needs it only when these entry
// points are called; a process that has already loaded an NCCL (PyTorch bundles one) shares that copy.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/onegpu_cuda.h"
#include "og_host.h"

using namespace og_host;

struct og_comm {
    og_device* device = nullptr;
    int nranks = 0, rank = 0;
    ncclComm_t nccl = nullptr;
    void* staging = nullptr;  // root of a column gather: the other ranks' shards before they are put in place
    size_t staging_bytes = 0;
};

namespace {

const char* kComm = "Communicator";

struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) {
            api.why = "libnccl.so.2 could not be loaded";
            return;
        }
        auto sym = [&](const char* name) { return dlsym(h, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
        api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.group_start && api.group_end &&
                 api.send && api.recv && api.all_gather && api.error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks an entry point this library calls";
    });
    return api;
}

const NcclApi& need_nccl() {
    const NcclApi& api = nccl();
    if (!api.ok) unsupported(kComm, api.why, "NCCL", "libnccl.so.2 (NCCL 2.x)", "absent");
    return api;
}

void check_nccl(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return;
    const NcclApi& api = nccl();
    throw OgError{OG_ERROR_CUDA, kComm, "", std::string(what) + ": NCCL " + (api.error_string ? api.error_string(r) : "error"),
                  "", "", ""};
}

// The column shards of a gathered result, as the placement kernel reads them.
constexpr int kMaxPlaceRanks = 64;
struct Placement {
    const uint8_t* src[kMaxPlaceRanks];  // shard of rank r: rows of width[r] bytes, dense
    int64_t col0[kMaxPlaceRanks];        // its first byte within an output row
    int64_t width[kMaxPlaceRanks];       // bytes per row
    int nranks;
    int64_t row_bytes;                   // of the output
    int64_t rows;
    int vec;                             // every offset and width is a multiple of 16 bytes
};

// Puts the shards in place: output row i is the concatenation of row i of every shard. One CTA per row (grid-stride
// over rows), consecutive threads on consecutive 16-byte words, so every read and write is coalesced.
__global__ void __launch_bounds__(256) place_columns_kernel(const __grid_constant__ Placement pl, uint8_t* out) {
    for (int64_t row = blockIdx.x; row < pl.rows; row += gridDim.x) {
        uint8_t* dst = out + row * pl.row_bytes;
        for (int r = 0; r < pl.nranks; r++) {
            const int64_t w = pl.width[r];
            const uint8_t* src = pl.src[r] + row * w;
            if (pl.vec) {
                for (int64_t j = threadIdx.x * 16; j < w; j += 256 * 16)
                    *reinterpret_cast<uint4*>(dst + pl.col0[r] + j) = __ldcs(reinterpret_cast<const uint4*>(src + j));
            } else {
                for (int64_t j = threadIdx.x; j < w; j += 256) dst[pl.col0[r] + j] = src[j];
            }
        }
    }
}

og_comm* live(og_comm* c) {
    if (c == nullptr || c->nccl == nullptr)
        throw OgError{OG_ERROR_INVALID_HANDLE, kComm, "comm", "null communicator", "", "", ""};
    return c;
}

}  // namespace

extern "C" {

OG_API og_status og_comm_unique_id(uint8_t* id) {
    return guard([&] {
        if (id == nullptr) null_arg(kComm, "id");
        const NcclApi& api = need_nccl();
        ncclUniqueId u;
        check_nccl(api.get_unique_id(&u), "ncclGetUniqueId");
        static_assert(sizeof(u) == OG_COMM_ID_BYTES, "the id is NCCL's unique id");
        std::memcpy(id, &u, sizeof(u));
    });
}

OG_API og_status og_comm_create(og_device* device, int32_t nranks, int32_t rank, const uint8_t* id, og_comm** out) {
    return guard([&] {
        if (device == nullptr) null_arg(kComm, "device");
        if (id == nullptr) null_arg(kComm, "id");
        if (out == nullptr) null_arg(kComm, "out");
        *out = nullptr;
        if (nranks < 1) shape(kComm, "nranks", "must be at least 1, got " + std::to_string(nranks));
        if (rank < 0 || rank >= nranks)
            shape(kComm, "rank", std::to_string(rank) + " is outside [0, " + std::to_string(nranks) + ")");
        const NcclApi& api = need_nccl();
        use(device);
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof(u));
        auto* c = new og_comm();
        c->device = device;
        c->nranks = nranks;
        c->rank = rank;
        const ncclResult_t r = api.comm_init_rank(&c->nccl, nranks, u, rank);
        if (r != ncclSuccess) {
            delete c;
            check_nccl(r, "ncclCommInitRank");
        }
        *out = c;
    });
}

OG_API og_status og_comm_destroy(og_comm* comm) {
    return guard([&] {
        if (comm == nullptr) return;
        use(comm->device);
        cudaStreamSynchronize(comm->device->stream);
        if (comm->nccl != nullptr) nccl().comm_destroy(comm->nccl);
        if (comm->staging != nullptr) cudaFree(comm->staging);
        delete comm;
    });
}

OG_API og_status og_comm_gather_columns(og_comm* comm, const void* shard, int32_t elem_bytes, int32_t batch, int32_t m,
                                        const int32_t* widths, void* out, int32_t root) {
    return guard([&] {
        live(comm);
        if (widths == nullptr) null_arg(kComm, "widths");
        if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
            shape(kComm, "elemBytes", "must be 1, 2, 4 or 8, got " + std::to_string(elem_bytes));
        if (batch < 1) shape(kComm, "batch", "must be at least 1, got " + std::to_string(batch));
        if (m < 0) shape(kComm, "m", "must not be negative, got " + std::to_string(m));
        if (comm->nranks > kMaxPlaceRanks)
            unsupported(kComm, "a column gather over more than 64 ranks", "Ranks", "at most 64",
                        std::to_string(comm->nranks));
        if (root < 0 || root >= comm->nranks)
            shape(kComm, "root", std::to_string(root) + " is outside [0, " + std::to_string(comm->nranks) + ")");
        int64_t n = 0;
        std::vector<int64_t> col0(comm->nranks);
        for (int r = 0; r < comm->nranks; r++) {
            if (widths[r] < 0) shape(kComm, "widths", "width of rank " + std::to_string(r) + " is negative");
            col0[r] = n;
            n += widths[r];
        }
        const int64_t rows = int64_t(batch) * m;
        const int64_t mine = rows * widths[comm->rank] * elem_bytes;
        if (mine > 0 && shard == nullptr) null_arg(kComm, "shard");
        if (comm->rank == root && rows * n > 0 && out == nullptr) null_arg(kComm, "out");
        if (rows == 0 || n == 0) return;
        const NcclApi& api = nccl();
        use(comm->device);
        cudaStream_t s = comm->device->stream;
        if (comm->rank != root) {
            if (mine > 0) check_nccl(api.send(shard, size_t(mine), ncclChar, root, comm->nccl, s), "ncclSend");
            return;
        }
        // Root: receive every other shard into the staging buffer, then put each one (and its own) in place with one
        // kernel: shard r's row i lands at columns [col0[r], col0[r] + widths[r]) of output row i.
        std::vector<int64_t> at(comm->nranks, 0);
        int64_t need = 0;
        for (int r = 0; r < comm->nranks; r++) {
            if (r == root) continue;
            at[r] = need;
            need += (rows * widths[r] * elem_bytes + 255) & ~int64_t(255);
        }
        if (size_t(need) > comm->staging_bytes) {
            if (comm->staging != nullptr) {
                check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
                check_cuda(cudaFree(comm->staging), "gather staging");
                comm->staging = nullptr;
                comm->staging_bytes = 0;
            }
            check_cuda(cudaMalloc(&comm->staging, size_t(need)), "gather staging");
            comm->staging_bytes = size_t(need);
        }
        uint8_t* stage = static_cast<uint8_t*>(comm->staging);
        check_nccl(api.group_start(), "ncclGroupStart");
        for (int r = 0; r < comm->nranks; r++) {
            if (r == root || widths[r] == 0) continue;
            const ncclResult_t e = api.recv(stage + at[r], size_t(rows * widths[r] * elem_bytes), ncclChar, r,
                                            comm->nccl, s);
            if (e != ncclSuccess) {
                api.group_end();
                check_nccl(e, "ncclRecv");
            }
        }
        check_nccl(api.group_end(), "ncclGroupEnd");
        Placement pl = {};
        pl.nranks = comm->nranks;
        pl.row_bytes = n * elem_bytes;
        pl.rows = rows;
        bool vec = (reinterpret_cast<uintptr_t>(out) & 15) == 0 && (pl.row_bytes & 15) == 0;
        for (int r = 0; r < comm->nranks; r++) {
            pl.src[r] = static_cast<const uint8_t*>(r == root ? shard : stage + at[r]);
            pl.col0[r] = col0[r] * elem_bytes;
            pl.width[r] = int64_t(widths[r]) * elem_bytes;
            vec = vec && (reinterpret_cast<uintptr_t>(pl.src[r]) & 15) == 0 && (pl.col0[r] & 15) == 0 &&
                  (pl.width[r] & 15) == 0;
        }
        pl.vec = vec ? 1 : 0;
        const int grid = static_cast<int>(std::min<int64_t>(rows, int64_t(comm->device->sm_count) * 8));
        place_columns_kernel<<<grid, 256, 0, s>>>(pl, static_cast<uint8_t*>(out));
        check_cuda(cudaGetLastError(), "gather placement");
    });
}

OG_API og_status og_comm_all_gather(og_comm* comm, const void* send, uint64_t bytes, void* recv) {
    return guard([&] {
        live(comm);
        if (bytes == 0) return;
        if (send == nullptr) null_arg(kComm, "send");
        if (recv == nullptr) null_arg(kComm, "recv");
        use(comm->device);
        check_nccl(nccl().all_gather(send, recv, size_t(bytes), ncclChar, comm->nccl, comm->device->stream),
                   "ncclAllGather");
    });
}

}  // extern "C"
