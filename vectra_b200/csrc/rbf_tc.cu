// rbf_tc.cu: tensor-core (tcgen05 + TMEM) path for long sequences.
// Until the tensor-core kernel is in place every problem goes to the
// generic kernel; tc_supports declines all of them.
#include "rbf_common.cuh"

namespace vectra {

bool tc_supports(const RbfProblem& p) {
  (void)p;
  return false;
}

cudaError_t launch_tc(const RbfProblem& p, cudaStream_t stream) {
  (void)p;
  (void)stream;
  return cudaErrorNotSupported;
}

}  // namespace vectra
