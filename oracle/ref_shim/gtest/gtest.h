// Compile-only stand-in for GoogleTest, used when the reference's test
// sources are compiled in place to reach their CPU helper functions
// (compute_expected_*). It is test infrastructure, not product code.
//
// TEST(...) bodies become unused static functions: they are type-checked
// but never registered, called or emitted. The ASSERT_* macros keep the
// "ASSERT_X(a, b) << message" streaming syntax compiling.
#pragma once

#include <cmath>

namespace ref_shim
{
struct Message
{
    template <typename V>
    Message &operator<<(const V &) { return *this; }
};
struct Failure
{
    void operator=(const Message &) const {}
};
} // namespace ref_shim

#define REF_SHIM_CHECK(cond) \
    if (cond)                \
        ;                    \
    else                     \
        return ::ref_shim::Failure() = ::ref_shim::Message()

#define TEST(suite, name) [[maybe_unused]] static void ref_shim_unused_##suite##_##name()
#define ASSERT_EQ(a, b) REF_SHIM_CHECK((a) == (b))
#define ASSERT_NE(a, b) REF_SHIM_CHECK((a) != (b))
#define ASSERT_TRUE(c) REF_SHIM_CHECK(c)
#define ASSERT_FALSE(c) REF_SHIM_CHECK(!(c))
#define ASSERT_NEAR(a, b, tol) REF_SHIM_CHECK(std::fabs((a) - (b)) <= (tol))
#define EXPECT_EQ ASSERT_EQ
#define EXPECT_NEAR ASSERT_NEAR
