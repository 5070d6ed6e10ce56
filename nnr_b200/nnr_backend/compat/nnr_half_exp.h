// Forced include for nnr's Sigmoid.cpp only, when nnr is built with GCC 13,
// which rejects that file's bf16/fp16 lambda: its two branches deduce
// float16_t and double; these overloads make exp() of a half
// type return the half type, so both branches agree. With std::exp visible
// beside them, float and double keep their own overloads.
#pragma once
#include <cmath>
#include "float16.h"
#include "bfloat16.h"
using std::exp;
inline float16_t exp(float16_t v) { return float16_t(std::exp((float)v)); }
inline bfloat16_t exp(bfloat16_t v) { return bfloat16_t(std::exp((float)v)); }
