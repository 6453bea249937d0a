// Stand-in for tinygs/include/tinygs/utils/scope_timer.hpp, which the
// reference's rasterizer forward includes but does not use.
#pragma once
