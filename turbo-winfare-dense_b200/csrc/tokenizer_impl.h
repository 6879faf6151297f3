// The body of g4dense::Tokenizer (include/g4dense/tokenizer.hpp), shared by the C++ API files.
#pragma once
#include "g4dense/tokenizer.hpp"
#include "tokenizer.h"

namespace g4dense {
struct Tokenizer::Impl {
    g4b::Tokenizer t;
};
}  // namespace g4dense
