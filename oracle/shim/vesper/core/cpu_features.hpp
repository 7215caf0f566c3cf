#pragma once
// Build shim for compiling the reference IVF-PQ sources as the oracle.
//
// The reference includes "vesper/core/cpu_features.hpp" (src/index/ivf_pq.cpp:19)
// and calls vesper::core::decide_use_avx512_from_env_and_cpu() when it configures
// FastScanPq (src/index/ivf_pq.cpp:2462,4647,4816), but the header is absent from
// the reference tree.  This file supplies the two functions it needs.  The oracle is
// compiled without -mavx512f (the reference's AVX-512 build does not compile), so the
// AVX-512 FastScan path can never be selected and both functions report false unless
// the translation unit was built with AVX-512 enabled.
#include <cstdlib>

namespace vesper::core {

inline bool cpu_supports_avx512_runtime() noexcept {
#if defined(__AVX512F__) && (defined(__GNUC__) || defined(__clang__))
    return __builtin_cpu_supports("avx512f");
#else
    return false;
#endif
}

inline bool decide_use_avx512_from_env_and_cpu() noexcept {
#if defined(__AVX512F__)
    const char* v = std::getenv("VESPER_AVX512");
    if (v && v[0] == '0') return false;
    return cpu_supports_avx512_runtime();
#else
    return false;
#endif
}

}  // namespace vesper::core
