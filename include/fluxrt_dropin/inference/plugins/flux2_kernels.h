// Drop-in for fluxrt-cpp's src/inference/plugins/flux2_kernels.h: the declarations of that header, implemented by libfxr.so.
#pragma once
#include "fxr_reference_api.h"
