// The reference's benchmark driver (benchmark.cpp, compiled unchanged from
// the reference checkout) linked against libnerf_b200.so -- the drop-in check
// of the nerf.h boundary.  Test infrastructure only.
//
// benchmark.cpp is C++23 with `import std;`, which GCC 13 cannot compile
// (no standard-library module).  This translation unit first includes every
// header the driver would see -- the standard library, nerf.h, the stb-API
// PNG shims over the library's own codec, nlohmann::json -- and then turns
// the driver's `import std;` line into a harmless namespace alias before
// including the driver's source as it lies.  Every header it includes again
// is skipped by its include guard, so the macro touches only the driver's own
// text, whose single use of the word is that line.
#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <limits>
#include <memory>
#include <numeric>
#include <span>
#include <sstream>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

#include "nerf.h"
#include "stb/stb_image.h"
#include "stb/stb_image_write.h"
#include "json/json.hpp"

#define import namespace nerf_b200_import_std_shim =
#include "benchmark.cpp"
#undef import
