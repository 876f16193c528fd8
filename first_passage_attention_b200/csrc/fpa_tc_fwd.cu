#include "fpa_tc.h"

namespace fpa {

bool tc_supports(int D) { return false; }

int tc_fwd(const FpaFwdArgs& a, const Dims& d, const Stats& st, int* status, cudaStream_t s, int* launched,
           std::string* err) {
  *launched = 0;
  *err = "tensor-core forward not built";
  return FPA_ERR_UNSUPPORTED;
}

}  // namespace fpa
