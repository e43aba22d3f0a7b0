// kvm_noalloc.cu -- kvm_quantize_rows_noalloc: the row-quantize kernel with
// its work list in a fixed device array instead of a cudaMalloc'd buffer.
//
// Who needs it: callers that must not allocate device memory while they run.
// For example, a runtime whose caching allocator already owns all free HBM
// (a raw cudaMalloc then fails or fragments it), or a latency-critical path
// that cannot afford the implicit device synchronisation of cudaMalloc /
// cudaFree.  kvm_quantize_rows allocates, uses and frees a small work list on
// every call, so those callers cannot use it.
//
// The work list lives in g_noalloc_scratch, a file-scope __device__ array of
// kNoallocMaxItems entries.  Every device that loads this library holds the
// array (about 192 KiB) until the process exits.  Host code cannot pass the
// array's name to a kernel -- on the host it is only a stand-in symbol -- so
// its device address is looked up once per device with cudaGetSymbolAddress,
// during the first call on that device (with that device current).  That
// first call should therefore happen before any stream capture begins.
#include <mutex>

#include "kvm_internal.cuh"
#include "kvm_kernels.h"

namespace kvm {
void set_sessionless_error(const char *msg);
namespace {

// Work items (one per row tile) the array can describe.
constexpr uint32_t kNoallocMaxItems = 16384;

// Layout (uint32 words): block ids [max], slots [max], rows per item [max],
// then the 2-entry destination pointer array (8-byte aligned).
constexpr uint32_t kNoallocPtrWord = 3u * kNoallocMaxItems;
constexpr uint32_t kNoallocWords = kNoallocPtrWord + 4u;

static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoallocWords];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
uint32_t *g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
cudaError_t noalloc_scratch(uint32_t **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = static_cast<uint32_t *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

// Identity work list: item i = rows [i*R, i*R + rows_i) written to slot i.
// Every word the quantize launch reads is rewritten here, so nothing left by
// an earlier call is used.
__global__ void noalloc_fill_kernel(uint32_t *w, uint32_t n_items, uint64_t n_rows, uint32_t R,
                                    uint8_t *dst) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_items;
         i += gridDim.x * blockDim.x) {
        w[i] = i;
        w[kNoallocMaxItems + i] = i;
        const uint64_t left = n_rows - static_cast<uint64_t>(i) * R;
        w[2u * kNoallocMaxItems + i] = static_cast<uint32_t>(left < R ? left : R);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        uint8_t **ptrs = reinterpret_cast<uint8_t **>(w + kNoallocPtrWord);
        ptrs[0] = dst;
        ptrs[1] = dst;
    }
}

}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" kvm_status kvm_quantize_rows_noalloc(kvm_stream stream, int32_t type, const void *d_src,
                                                uint64_t n_rows, uint32_t n_embd, void *d_dst) {
    const bool type_ok = type == KVM_TYPE_F16 || type == KVM_TYPE_Q8_0 ||
                         type == KVM_TYPE_Q4_0 || type == KVM_TYPE_Q5_0;
    if (!type_ok || n_embd == 0 || n_embd % 32u != 0 || n_embd > 16384u) return KVM_EINVAL;
    if (n_rows == 0) return KVM_OK;
    if (!d_src || !d_dst || (reinterpret_cast<uintptr_t>(d_src) & 15u)) return KVM_EINVAL;
    if (reinterpret_cast<uintptr_t>(d_dst) & 1u) {
        set_sessionless_error("kvm_quantize_rows_noalloc: d_dst must be 2-byte aligned");
        return KVM_EINVAL;
    }
    const uint32_t R = stagein_rows_per_tile(n_embd, 128u);
    const uint64_t n_items64 = (n_rows + R - 1) / R;
    if (n_items64 > kNoallocMaxItems) {
        set_sessionless_error("kvm_quantize_rows_noalloc: more than 16384 row tiles "
                              "(rows_per_tile = 8192 / n_embd, at most 128); split the call");
        return KVM_EINVAL;
    }
    const uint32_t n_items = static_cast<uint32_t>(n_items64);
    uint32_t *w = nullptr;
    if (noalloc_scratch(&w) != cudaSuccess) {
        set_sessionless_error("kvm_quantize_rows_noalloc: cudaGetSymbolAddress failed");
        return KVM_ECUDA;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    noalloc_fill_kernel<<<(n_items + 255u) / 256u, 256, 0, st>>>(w, n_items, n_rows, R,
                                                                  static_cast<uint8_t *>(d_dst));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_sessionless_error(cudaGetErrorString(e));
        return KVM_ECUDA;
    }
    const uint32_t rb = static_cast<uint32_t>(kvm_row_bytes(type, n_embd));
    StageinArgs a{};
    a.cold_block = w;
    a.cold_to = reinterpret_cast<const int32_t *>(w + kNoallocMaxItems);
    a.n_items_dev = nullptr;
    a.n_items_host = n_items;
    a.item0 = 0;
    a.max_items = n_items;
    a.src_by_item = 1;
    a.n_kv = 1;
    a.src_k = static_cast<const uint8_t *>(d_src);
    a.src_v = static_cast<const uint8_t *>(d_src);
    a.layer_stride = 0;
    a.item_stride = static_cast<uint64_t>(R) * n_embd * 2u;
    a.row_stride = 2ull * n_embd;
    a.n_tokens = w + 2u * kNoallocMaxItems;
    a.max_blocks = n_items;
    a.dst_k = reinterpret_cast<uint8_t *const *>(w + kNoallocPtrWord);
    a.dst_v = a.dst_k;
    a.n_layer = 1;
    a.block_tokens = R;
    a.n_embd = n_embd;
    a.n_slots = n_items;
    a.type_k = type;
    a.type_v = type;
    a.row_bytes_k = rb;
    a.row_bytes_v = rb;
    a.rows_per_tile = R;
    a.tile_in_bytes = R * n_embd * 2u;
    a.tile_out_bytes = (R * rb + 15u) & ~15u;
    a.bulk_store = (rb % 16u == 0 && (reinterpret_cast<uintptr_t>(d_dst) & 15u) == 0) ? 1u : 0u;
    a.status = nullptr;        // no host wait: a wait timeout inside is not reported
    e = launch_stagein(a, st, 0);
    if (e != cudaSuccess) {
        set_sessionless_error(cudaGetErrorString(e));
        return KVM_ECUDA;
    }
    return KVM_OK;
}
