// Device-side include of the W4A16 tensor-core GEMV (mma_gemv.cu); the host API is in api.h.
#pragma once
#include "common.cuh"
#include "api.h"
