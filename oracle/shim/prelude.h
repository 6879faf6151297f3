// Force-included before every reference translation unit built into oracle/_ref.
//
// TEST INFRASTRUCTURE ONLY: this lets the reference's own CPU oracle
// (src/cpu_reference.cpp) compile unmodified on Linux so it can serve as the
// parity checker. Nothing in the product links it.
//
// The reference maps the container only under _WIN32 (src/cpu_reference.cpp:197-235);
// its POSIX branch reads the header and leaves the mapping null, so
// forward_single_token would dereference nullptr. We therefore parse the C++
// standard library first (so libstdc++'s own _WIN32 checks see a Linux build) and
// only then define _WIN32, which routes the reference's #ifdef _WIN32 blocks to the
// POSIX stand-ins in shim/windows.h.
#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <functional>
#include <iostream>
#include <map>
#include <memory>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>
#define _WIN32 1
