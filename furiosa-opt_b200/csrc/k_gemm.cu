// Tensor-core GEMM for the plain-GEMM contractions (placeholder until the tcgen05 kernel lands):
// returns false so the generic per-cell contraction runs.
#include "ctx.hpp"

namespace fopt {

bool launch_gemm_tc(fopt_ctx*, void*, int, const void*, const void*, int, int64_t, int64_t, int64_t, int64_t, int64_t,
                    int64_t, const fopt_epilogue*, const float*, int) {
  return false;
}

}  // namespace fopt
