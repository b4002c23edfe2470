// Drop-in for fluxrt-cpp's src/inference/kernels/spatial_kv_cache.h: the declarations of that header, implemented by libfxr.so.
#pragma once
#include "fxr_reference_api.h"
