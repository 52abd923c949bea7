// bitwidth_benchmark_core.hpp -- the reference's header name for aut/bitwidth.hpp.
//
// Code written against the reference (include/bitwidth_benchmark_core.hpp) includes "bitwidth_benchmark_core.hpp" with
// -I<this directory> and gets the same names from this library.
#ifndef AUT_FWD_BITWIDTH_BENCHMARK_CORE_HPP_
#define AUT_FWD_BITWIDTH_BENCHMARK_CORE_HPP_
#include "aut/bitwidth.hpp"
#endif
