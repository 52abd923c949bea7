// memory_accessor.hpp -- the reference's header name for aut/memory_accessor.hpp.
//
// Code written against the reference (include/memory_accessor.hpp) includes "memory_accessor.hpp" with
// -I<this directory> and gets the same names from this library.
#ifndef AUT_FWD_MEMORY_ACCESSOR_HPP_
#define AUT_FWD_MEMORY_ACCESSOR_HPP_
#include "aut/memory_accessor.hpp"
#endif
