// All kernels of libfastssim.so for sm_100a (one header per family).
#pragma once

#include "fssim_common.cuh"
#include "fssim_fused.cuh"
#include "fssim_forward.cuh"
#include "fssim_f64.cuh"
