// The reference's IncrementalDetokenizer and StreamingStopMatcher (include/g4dense/detokenizer.hpp
// of the reference; behaviour of src/detokenizer.cpp): streamed text never splits a UTF-8
// character and equals batch decoding; a stop string is never partly shown.
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

#include "g4dense/tokenizer.hpp"

namespace g4dense {

class G4DENSE_CXX_API IncrementalDetokenizer {
   public:
    // `tok` must outlive the detokenizer.
    explicit IncrementalDetokenizer(const Tokenizer& tok, bool skip_special = true);
    ~IncrementalDetokenizer();
    IncrementalDetokenizer(const IncrementalDetokenizer&) = delete;
    IncrementalDetokenizer& operator=(const IncrementalDetokenizer&) = delete;

    // Returns text that is now definitely complete.
    std::string push(uint32_t token);
    // Flushes anything still buffered.
    std::string finish();
    void reset();

   private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

class G4DENSE_CXX_API StreamingStopMatcher {
   public:
    StreamingStopMatcher();
    explicit StreamingStopMatcher(std::vector<std::string> stops);
    ~StreamingStopMatcher();
    StreamingStopMatcher(const StreamingStopMatcher& o);
    StreamingStopMatcher& operator=(const StreamingStopMatcher& o);

    // Returns the text that is safe to emit: everything before a matched stop, withholding a tail
    // that could still become one.
    std::string push(std::string_view text);
    std::string finish();

    bool stopped() const;
    const std::string& matched() const;
    bool empty() const;

   private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace g4dense
