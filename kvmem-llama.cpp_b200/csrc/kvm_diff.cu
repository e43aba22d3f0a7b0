// kvm_diff.cu -- selection diff (KvMemPlan) and chronological window layout
// for a selection already in the plan (kvm_select_groups,
// kvm_set_selection_ids); after kvm_select the fused select + diff kernel
// of kvm_select.cu runs instead.  The body is diff_core (kvm_diff.cuh).
#include "kvm_diff.cuh"

namespace kvm {

__global__ void __launch_bounds__(kDiffThreads) diff_kernel(DiffArgs a) {
    extern __shared__ uint8_t fl[];
    const uint32_t n = a.n_blocks;
    diff_core(a, min(a.plan.hdr->n_selected, n), fl, fl + (n ? n : 1u), false);
}

// kvm_reset_window on its own (when no diff absorbs it): nothing in the
// working set, GPU-tier blocks drop to the CPU tier, no window slots.
__global__ void reset_window_kernel(BlockTable bt, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        bt.in_ws[i] = 0;
        if (bt.tier[i] == KVM_TIER_GPU) bt.tier[i] = KVM_TIER_CPU;
        bt.gpu_slot[i] = -1;
    }
}

cudaError_t launch_reset_window(const BlockTable &bt, uint32_t n, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    reset_window_kernel<<<(n + 255u) / 256u < 1024u ? (n + 255u) / 256u : 1024u, 256, 0, stream>>>(bt, n);
    return cudaGetLastError();
}

cudaError_t launch_diff(const DiffArgs &a, cudaStream_t stream) {
    const size_t smem = 2u * (a.n_blocks ? a.n_blocks : 1u);
    if (smem > 48u * 1024u)
        cudaFuncSetAttribute(diff_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    diff_kernel<<<1, kDiffThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace kvm
