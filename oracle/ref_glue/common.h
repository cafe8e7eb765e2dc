// Shared helpers for the glue translation units that expose the reference's
// CPU test helpers (compiled from the reference's own test sources, in
// place) through a C ABI. Test infrastructure only.
#pragma once
#include <cstdint>
#include <cstring>
#include <vector>

template <typename V>
static std::vector<V> ref_glue_vec(const V *p, size_t n) { return std::vector<V>(p, p + n); }

template <typename V>
static void ref_glue_out(const std::vector<V> &v, V *p) { std::memcpy(p, v.data(), v.size() * sizeof(V)); }
