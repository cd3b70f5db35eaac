// Host helpers shared by the translation units of the single-head
// operators (head_ops.cu, integrate.cu).
#pragma once
#include "abi.h"
#include "head_ops.cuh"

namespace gfn_head_ops {
using namespace gfn;
using namespace gfn_abi;


constexpr int kMaxHeadDim = 256;  // 8 elements per lane
constexpr size_t kMaxSmem = 220 * 1024;

inline int epl_for(int hd) { return hd <= 32 ? 1 : hd <= 64 ? 2 : hd <= 128 ? 4 : 8; }

inline size_t smem_bytes(int hd, int rank, int fin, bool fric, bool igate) {
  return (size_t)hops::smem_layout(hd, rank, fin, fric, igate).total * 4;
}

inline int check_common(const char* what, int batch, int dim, int rank, int topology, float plasticity, float R,
                 float r) {
  if (batch < 0 || dim <= 0) return fail(GFN_ERR_INVALID, "%s: batch=%d dim=%d", what, batch, dim);
  if (dim > kMaxHeadDim) return fail(GFN_ERR_UNSUPPORTED, "%s: head dim %d > %d", what, dim, kMaxHeadDim);
  if (topology != 0 && topology != 1) return fail(GFN_ERR_UNSUPPORTED, "%s: topology %d", what, topology);
  if (plasticity != 0.f) return fail(GFN_ERR_UNSUPPORTED, "%s: plasticity", what);
  if (topology == 0 && rank != 4 && rank != 8 && rank != 16)
    return fail(GFN_ERR_UNSUPPORTED, "%s: rank %d not in {4, 8, 16}", what, rank);
  if (topology == 1 && !(r != 0.f)) return fail(GFN_ERR_INVALID, "%s: minor radius 0", what);
  (void)R;
  return GFN_OK;
}

// Dispatch on (rank, elements per lane); the toroidal path ignores the rank
// (it runs the rank-4 instance with no U / W).
template <template <int, int> class K, typename... Args>
int dispatch(int rank, int hd, Args&&... args) {
  const int epl = epl_for(hd);
  const int rk = rank == 8 ? 8 : rank == 16 ? 16 : 4;
#define GFN_HO(RK, EPL) \
  if (rk == RK && epl == EPL) return K<RK, EPL>::run(args...);
#define GFN_HOR(RK) GFN_HO(RK, 1) GFN_HO(RK, 2) GFN_HO(RK, 4) GFN_HO(RK, 8)
  GFN_HOR(4) GFN_HOR(8) GFN_HOR(16)
#undef GFN_HOR
#undef GFN_HO
  return fail(GFN_ERR_UNSUPPORTED, "head op: rank %d / dim %d", rank, hd);
}

}  // namespace gfn_head_ops
