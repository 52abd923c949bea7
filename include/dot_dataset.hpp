// dot_dataset.hpp -- the reference's header name for aut/dot_dataset.hpp.
//
// Code written against the reference (include/dot_dataset.hpp) includes
// "dot_dataset.hpp" with -I<this directory> and gets the same names from this
// library.
#ifndef AUT_FWD_DOT_DATASET_HPP_
#define AUT_FWD_DOT_DATASET_HPP_
#include "aut/dot_dataset.hpp"
#endif
