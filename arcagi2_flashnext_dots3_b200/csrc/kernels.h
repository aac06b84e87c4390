// Declarations shared by the CUDA-core kernels (kernels.cu and friends) and the bindings.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
