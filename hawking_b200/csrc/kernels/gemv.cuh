// Small-batch dequant GEMV (see gemv.cu); declarations live in api.h.
#pragma once
#include "qformats.cuh"
