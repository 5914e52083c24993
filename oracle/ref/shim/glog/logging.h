// Minimal stand-in for glog's CHECK used by the reference's lotus_utils.hpp
// (glog is not installed here).  Test infrastructure only: lets the
// reference's operator sources compile unchanged into oracle/_ref/.
#pragma once
#include <cstdlib>
#include <iostream>

namespace lotus_ref_shim {
struct Fatal {
  bool ok;
  ~Fatal() {
    if (!ok) {
      std::cerr << std::endl;
      std::abort();
    }
  }
  template <class T>
  Fatal& operator<<(const T& v) {
    if (!ok) std::cerr << v;
    return *this;
  }
};
}  // namespace lotus_ref_shim

#define CHECK(cond) lotus_ref_shim::Fatal{static_cast<bool>(cond)}
