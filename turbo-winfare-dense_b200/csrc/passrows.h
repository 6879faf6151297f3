// Row limits of one forward pass, shared by host and device code.
#pragma once

namespace g4b {

constexpr int kMaxM = 16;          // rows of a verify pass (B-frag layout)
constexpr int kPrefillRows = 128;  // rows of a prefill pass (wide layout)

}  // namespace g4b
