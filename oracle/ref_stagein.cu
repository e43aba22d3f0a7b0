// ref_stagein.cu -- TEST INFRASTRUCTURE ONLY.
//
// The reference's own stage-in device kernels -- fwht_kernel<N>, quant_q8_0,
// quant_q4_0 and rope_neox_kernel of src/adapter/llama-kvmem-stagein.cu
// (:16-30 block layouts, :104-130, :159-178, :180-233) -- compiled unchanged
// with nvcc's default floating point, as the reference's CMake compiles that
// file into the llama target (no fast math; multiply-adds may be contracted).
// oracle/Makefile cuts their text out of the reference file at build time
// into _ref/stagein_kernels.inc, a temporary that make deletes after the
// link.  The launch wrappers below are this repository's; they use the
// reference's launch shapes (llama-kvmem-stagein.cu:526-530, :549-575,
// :577-604).  GPU tests compare the CPU oracle with these kernels.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

namespace {
#include "stagein_kernels.inc"
}  // namespace

extern "C" {

// In place on n_rows rows of nrot floats (device memory): scale by
// 1/sqrtf(nrot), then the butterflies.  Returns a cudaError_t value.
int ref_cuda_fwht(float *d_x, int64_t n_rows, int nrot, cudaStream_t st) {
    const float scale = 1.0f / sqrtf(static_cast<float>(nrot));
    const int threads = 128;
    const int blocks = static_cast<int>((n_rows + threads - 1) / threads);
    switch (nrot) {
        case 64: fwht_kernel<64><<<blocks, threads, 0, st>>>(d_x, n_rows, scale); break;
        case 128: fwht_kernel<128><<<blocks, threads, 0, st>>>(d_x, n_rows, scale); break;
        case 256: fwht_kernel<256><<<blocks, threads, 0, st>>>(d_x, n_rows, scale); break;
        case 512: fwht_kernel<512><<<blocks, threads, 0, st>>>(d_x, n_rows, scale); break;
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
    return static_cast<int>(cudaGetLastError());
}

// n_blocks blocks of 32 floats to q8_0 (type 8, 34 bytes a block) or q4_0
// (type 2, 18 bytes a block) at d_y.  Returns a cudaError_t value.
int ref_cuda_quantize(int type, const float *d_x, void *d_y, int64_t n_blocks, cudaStream_t st) {
    const int threads = 256;
    const int blocks = static_cast<int>((n_blocks + threads - 1) / threads);
    if (type == 8) {
        quant_q8_0<<<blocks, threads, 0, st>>>(d_x, static_cast<block_q8_0 *>(d_y), n_blocks);
    } else if (type == 2) {
        quant_q4_0<<<blocks, threads, 0, st>>>(d_x, static_cast<block_q4_0 *>(d_y), n_blocks);
    } else {
        return static_cast<int>(cudaErrorInvalidValue);
    }
    return static_cast<int>(cudaGetLastError());
}

// NeoX RoPE in place on n_tokens rows of n_head x n_embd_head floats, pair
// (i, i + n_rot/2) turned by (pos0 + t) * d_theta[i].  Returns a cudaError_t.
int ref_cuda_rope_neox(float *d_x, int64_t n_tokens, int n_head, int n_embd_head, int n_rot,
                       int32_t pos0, const float *d_theta, cudaStream_t st) {
    const int threads = 64;
    const dim3 grid(static_cast<unsigned>((n_tokens + threads - 1) / threads), static_cast<unsigned>(n_head), 1);
    rope_neox_kernel<<<grid, threads, 0, st>>>(d_x, n_tokens, n_head, n_embd_head, n_rot, pos0, d_theta);
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
