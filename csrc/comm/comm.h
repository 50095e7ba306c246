// Host interface of the fused communication kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
