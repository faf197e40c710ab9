// compat/model.h — the reference's "model.h" name for callers that compile unchanged
// against librbk: put include/rubidium/compat first on the include path and
// "#include \"model.h\"" (src/main.cpp:5) resolves here.  Brings the drop-in types into
// the global namespace and supplies what the reference trainer takes from
// src/cuda_kernels.cuh: the CE check macro for the caller's own CUDA calls
// (cuda_kernels.cuh:13-14: print and exit on failure) and init_handles /
// destroy_handles (cuda_kernels.cuh:30-31), which have nothing to set up here:
// librbk holds no global cuBLAS / cuDNN handles.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "../model.h"

#ifndef CE
#define CE(e)                                                                                 \
    do {                                                                                      \
        cudaError_t rbk_ce_err_ = (e);                                                        \
        if (rbk_ce_err_ != cudaSuccess) {                                                     \
            fprintf(stderr, "CUDA %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(rbk_ce_err_)); \
            exit(1);                                                                          \
        }                                                                                     \
    } while (0)
#endif

inline void init_handles() {}
inline void destroy_handles() {}

using rubidium::LoRAConfig;
using rubidium::ModelConfig;
using rubidium::RubidiumTransformer;
