// Decode-path kernels (see decode_ops.cu, attention.cu); declarations live in api.h.
#pragma once
#include "common.cuh"
#include "qformats.cuh"
