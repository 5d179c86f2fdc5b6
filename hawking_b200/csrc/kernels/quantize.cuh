// GPU quantisers (see quantize.cu); declarations live in api.h.
#pragma once
#include "qformats.cuh"
