/* Forced-include shim for compiling the reference's main.cpp with g++ 13 / libstdc++ 13.
 * The reference calls std::fabsf, std::floorf, std::roundf and std::nearbyintf, which
 * libstdc++ 13 does not declare in namespace std (MSVC's STL does). This header only
 * re-exports the C library functions; the reference source is compiled unmodified.
 * Test infrastructure: only the oracle build uses it. */
#pragma once
#include <cmath>
#include <math.h>
namespace std { using ::fabsf; using ::floorf; using ::roundf; using ::nearbyintf; }
