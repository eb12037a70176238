// Kernels of the synchronous host-buffer call (m1moe_cuda_moe_layer_host):
// the caller's inputs come from, and the results go to, mapped pinned host
// memory through ordinary loads and stores, and the call ends with a sequence
// number stored to host memory that the host thread polls.  Copy-engine
// operations cost several microseconds each on the stream for these few KB,
// and a stream synchronisation adds a few more; these kernels chain to the
// layer kernel with programmatic dependent launch instead.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "pipeline.cuh"

namespace m1 {

// One float4 per thread, every load in flight at once (each costs a PCIe
// round trip).  Launched as the first node, without a programmatic edge, so
// it starts after everything before it on the stream; it lets the layer
// kernel launch at once (its prologue reads only constants).
__global__ void __launch_bounds__(256) k_stage_in(const float4 *__restrict__ host, float4 *__restrict__ dev,
                                                  int n4) {
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n4) dev[i] = host[i];
}

// After the layer (griddepcontrol.wait): out, indices and weights to host
// memory, then, once every store is visible system-wide, the next sequence
// number to the host's flag word.  One CTA; the stores are posted writes.
__global__ void __launch_bounds__(1024) k_stage_out(const float4 *__restrict__ dev, float4 *host, int n4,
                                                    unsigned *dseq, unsigned *hflag) {
    pdl_wait();
    for (int i = threadIdx.x; i < n4; i += blockDim.x) host[i] = dev[i];
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned v = *dseq + 1u;
        *dseq = v;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(hflag), "r"(v) : "memory");
    }
}

}  // namespace m1
