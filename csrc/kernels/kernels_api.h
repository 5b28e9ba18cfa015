// Host API of the elementwise / normalisation / loss / optimizer / codec
// kernels (SIMT sm_100a).  All launches are asynchronous on `stream`.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
