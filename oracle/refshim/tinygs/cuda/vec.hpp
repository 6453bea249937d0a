// Stand-in for tinygs/include/tinygs/cuda/vec.hpp: the reference's loss
// kernels include it but use none of its glm vector types.
#pragma once
#include "tinygs/common.hpp"
