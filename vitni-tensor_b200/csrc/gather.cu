// gather.cu -- completion side of the fused row-shard all-gather.
//
// A row-sharded linear (each rank owns a contiguous range of output rows,
// shard-invariant because every output row is its own reduction,
// vitni-tensor src/ops/quant.rs:1373-1377) writes its rows straight into the
// full-y buffer of every rank over NVLink and then adds 1 to every rank's
// arrival counter (kquant_matvec.cu). This kernel is the receiving side: it
// holds the stream until the expected number of arrivals has been seen, so
// that later work on the stream reads a complete y. Counters only grow; the
// number of arrivals consumed so far lives in device memory next to them, so
// the wait needs no host-side epoch and can be captured in a CUDA graph.
#include "vtq_device.cuh"
#include "vtq_internal.h"

namespace vtq {
namespace {

__global__ void gather_wait_kernel(const unsigned* cnt, unsigned* expected, unsigned signals,
                                   unsigned* status, uint64_t limit_ns) {
  // Programmatic launch: wait for this rank's gathered launches to finish,
  // let the next kernel start streaming its weights, then wait for the peers.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x != 0) return;
  const unsigned target = *expected + signals;
  const uint64_t t0 = globaltimer();
  for (;;) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
    if ((int)(v - target) >= 0) break;  // wrap-safe comparison
    if (globaltimer() - t0 > limit_ns) {
      // Give up: report, and count none of the missing arrivals as consumed.
      record_error(status, KERR_TIMEOUT);
      return;
    }
  }
  *expected = target;
  __threadfence_system();
}

}  // namespace

cudaError_t launch_gather_wait(unsigned* cnt, unsigned* expected, unsigned signals,
                               unsigned* status, cudaStream_t st, uint64_t limit_ns) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gather_wait_kernel, (const unsigned*)cnt, expected, signals,
                            status, limit_ns);
}

}  // namespace vtq
