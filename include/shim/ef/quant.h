// include/shim/ef/quant.h - stands in for the reference's include/ef/quant.h: the same API,
// running on the GPU through libefg.so (include/efg_ref_shim.hpp).
#pragma once
#include "../../efg_ref_shim.hpp"
