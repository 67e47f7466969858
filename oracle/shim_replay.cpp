// shim_replay.cpp -- the reference's training loop (train_replay.inc) running on this library's
// drop-in `ngp::cuda` layer (instant-ngp_b200/shim/ngp_train_cuda.cpp) instead of the reference's
// ngp.train.cu.  TEST INFRASTRUCTURE ONLY: built by `make -C oracle shim` against the reference's
// own ngp.train.h into oracle/_ref/libngp_shim_replay.so, loaded by tests/ and bench.py.
#include <algorithm>
#include <cstdio>
#include <exception>

#include <cuda_runtime.h>

#include "ngp.train.h"

namespace ref = ngp::cuda;
namespace cfg = ngp::cuda::config;

#include "train_replay.inc"
