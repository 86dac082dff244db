// Stand-in for the reference's npuSetup.hpp: the CPU AVX GEMV reads only the
// global verbosity level from it.
#pragma once
inline int debug_verbosity = 0;
