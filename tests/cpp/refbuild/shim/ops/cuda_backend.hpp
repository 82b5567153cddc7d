// Stand-in for the reference's include/ops/cuda_backend.hpp when its sources are built
// against the B200 library: the same interface, implemented by libib_cuda.so.
#pragma once
#include "ib_cuda_backend.hpp"
