// decoder_strategy_core.hpp -- the reference's header name for aut/decoder.hpp.
//
// Code written against the reference (include/decoder_strategy_core.hpp) includes "decoder_strategy_core.hpp" with
// -I<this directory> and gets the same names from this library.
#ifndef AUT_FWD_DECODER_STRATEGY_CORE_HPP_
#define AUT_FWD_DECODER_STRATEGY_CORE_HPP_
#include "aut/decoder.hpp"
#endif
