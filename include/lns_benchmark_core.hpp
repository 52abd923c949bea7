// lns_benchmark_core.hpp -- the reference's header name for aut/lns.hpp.
//
// Code written against the reference (include/lns_benchmark_core.hpp) includes "lns_benchmark_core.hpp" with
// -I<this directory> and gets the same names from this library.
#ifndef AUT_FWD_LNS_BENCHMARK_CORE_HPP_
#define AUT_FWD_LNS_BENCHMARK_CORE_HPP_
#include "aut/lns.hpp"
#endif
