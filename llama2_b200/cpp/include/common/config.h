// Semantic constants of the operator API (same values as the reference's
// include/common/config.h:3-16: they define the operators' results).
#pragma once

constexpr unsigned int WARP_SIZE = 32;
constexpr float SOFTMAX_EPS = 1e-6f;   // added to the softmax denominator
constexpr float RMSNORM_EPS = 1e-5f;   // added to mean(x^2)
constexpr float ROPE_BASE = 10000.f;   // theta_i = ROPE_BASE^(-2i/head_dim)
constexpr float TRAIN_SEQ_LEN = 4096.f; // RoPE length scaling starts above this
