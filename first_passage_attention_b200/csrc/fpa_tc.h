// Tensor-core (tcgen05 / TMEM / TMA) kernels for sm_100a.
#pragma once

#include <string>

#include "fpa_internal.h"

namespace fpa {

constexpr int kTcBT = 128;  // positions per tile of the tensor-core kernels (the MMA M and N)

bool tc_supports(int D);

// Forward pass on the tensor cores; `status` is the device status word of the workspace. Sets *launched to the
// number of kernels launched. Returns an FpaStatus; on failure writes a message into *err.
int tc_fwd(const FpaFwdArgs& a, const Dims& d, const Stats& st, const KeyCols& cols, int* status, cudaStream_t s,
           int* launched, std::string* err);

}  // namespace fpa
