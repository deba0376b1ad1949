// Tensor-core GEMM for sm_100a (tcgen05 + TMEM + TMA).  Placeholder until
// the tcgen05 kernel lands: reports "unsupported" so mmp_gemm falls back.
#include "mmp_internal.h"

namespace mmp {
int gemm_tc(int, int, long long, long long, long long, long long, const void *, long long, long long,
            const void *, long long, long long, void *, long long, long long) {
  return set_error(MMP_E_UNSUPPORTED, "tensor-core GEMM not built");
}
}  // namespace mmp
