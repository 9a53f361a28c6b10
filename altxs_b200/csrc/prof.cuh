// Launch accounting and optional per-kernel-class CUDA-event timing.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace altxs {

enum KernelClass : int {
    kKEmbed = 0,
    kKPrenorm,
    kKQmm,
    kKQkvPost,
    kKAttn,
    kKAttnMerge,
    kKPostAttn,
    kKFinal,
    kKCdfCode,
    kKCoder,
    kKTtt,
    kKFused,
    kKNumClasses
};

// Every kernel launch of the library goes through prof_begin/prof_end: the
// launch counter always counts; event pairs are recorded only while the
// profiler is enabled (altxs_profile(1)).
void prof_begin(cudaStream_t s, int cls);
void prof_end(cudaStream_t s);

}  // namespace altxs

#define ALTXS_LAUNCH(cls, stream, ...)         \
    do {                                       \
        ::altxs::prof_begin((stream), (cls));  \
        __VA_ARGS__;                           \
        ::altxs::prof_end((stream));           \
        ALTXS_LAUNCH_CHECK();                  \
    } while (0)
