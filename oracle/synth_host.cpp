// ORACLE BUILD — test infrastructure only.
//
// The package's synthetic-GGUF writer (fishai-engine_b200/csrc/synth.cpp and
// the quantisers it uses: host C++, no device code) compiled a second time,
// into oracle/build/libsynth.so, so that the CPU reference arm of bench.py
// writes its input file without loading the CUDA library.  Same sources and
// compiler flags as the package build: the two writers give byte-identical
// files (tests/test_cpu_product.py checks it).
#include "../fishai-engine_b200/csrc/fa_host.hpp"

namespace fa {
int synth_write(const char *path, const fa_synth_spec *s, uint64_t seed);
}

extern "C" int or_synth_write(const char *path, const fa_synth_spec *s, uint64_t seed) {
  return fa::synth_write(path, s, seed);
}

extern "C" size_t or_synth_last_error(char *buf, size_t cap) {
  const std::string &e = fa::last_error();
  if (buf && cap) {
    const size_t n = e.size() < cap - 1 ? e.size() : cap - 1;
    std::memcpy(buf, e.data(), n);
    buf[n] = 0;
  }
  return e.size();
}
