// Test infrastructure: lets the reference's own baseline/tests/boundaries.cpp
// compile unchanged against the C++ mirror of its API (include/gat_b200.hpp)
// and run on the B200 library (make -C oracle ref -> _ref/boundaries_on_b200).
// The reference's gat.hpp brings OpenMP and oneMKL along; the test sets their
// CPU thread counts, which have no meaning for the device library, so the two
// oneMKL setters are no-ops here.
#pragma once
#include <omp.h>

#include "gat_b200.hpp"

namespace gat = gat_b200;

inline void mkl_set_num_threads(int) {}
inline void mkl_set_dynamic(int) {}
