// Measurement entry points (not on the recurrence path).
#include "abi.h"
#include "latency_probe.cuh"

using namespace gfn;
using namespace gfn_abi;

namespace gfn_abi {
cudaError_t error_word_probe(int* v, int reset, cudaStream_t s) { return gfn_unit_error_word(v, reset, s); }
}  // namespace gfn_abi

extern "C" int gfn_debug_latency_probe(int rank, int clusters, int steps, long long* cycles,
                                       gfn_stream_t stream) {
  if (clusters < 1 || steps < 1 || !cycles) return fail(GFN_ERR_INVALID, "latency probe: bad arguments");
  void (*kern)(int, long long*) = nullptr;
  if (rank == 4) kern = latency_probe_kernel<4, 8>;
  else if (rank == 8) kern = latency_probe_kernel<8, 8>;
  else if (rank == 16) kern = latency_probe_kernel<16, 8>;
  else return fail(GFN_ERR_UNSUPPORTED, "latency probe: rank %d", rank);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 8;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)(8 * clusters));
  cfg.blockDim = dim3(32);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, steps, cycles), "latency probe launch");
}
