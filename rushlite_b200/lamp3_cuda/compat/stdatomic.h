// Stand-in for <stdatomic.h> when a C++ translation unit includes it.
// The reference's csrc/include/lamp3/tensor/cuda/memory.cuh:6 includes the C
// header but uses nothing from it; GCC 13 only makes that header valid C++
// from C++23 on, and the reference builds as C++20.  Listed first on the
// include path of lmpb's Lamp3 build (Makefile in this directory).
#pragma once
#include <atomic>
