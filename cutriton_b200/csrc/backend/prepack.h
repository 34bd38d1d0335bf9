#pragma once

// Constant preprocessing ("prepack") transforms.
//
// A kernel argument may name a prepack transform; the engine then runs the
// transform once on the host copy of the constant at upload time and binds
// the derived device tensor "<constant>::<prepack>" instead (e.g. convolution
// weights re-laid out K-major and split into TF32 hi/lo halves for the
// 3xTF32 tensor-core path). Transforms are pure host functions.

#include <cstdint>
#include <string>
#include <vector>

#include "cutriton/core/status.h"
#include "cutriton/core/tensor.h"

namespace cutriton {

std::string PrepackedName(const std::string& constant, const std::string& prepack);

// Applies the named transform to `data` (host bytes described by `desc`).
Status RunPrepack(const std::string& prepack, const TensorDesc& desc, const void* data,
                  TensorDesc* out_desc, std::vector<std::uint8_t>* out_bytes);

// True when `prepack` names a registered transform.
bool IsKnownPrepack(const std::string& prepack);

}  // namespace cutriton
