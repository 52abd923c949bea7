// storage_formats.hpp -- the reference's header name for aut/storage_formats.hpp.
//
// Code written against the reference (include/storage_formats.hpp) includes "storage_formats.hpp" with
// -I<this directory> and gets the same names from this library.
#ifndef AUT_FWD_STORAGE_FORMATS_HPP_
#define AUT_FWD_STORAGE_FORMATS_HPP_
#include "aut/storage_formats.hpp"
#endif
