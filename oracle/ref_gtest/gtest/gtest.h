// A small, runnable stand-in for the part of GoogleTest the reference's unit
// tests use (TEST, ASSERT_* / EXPECT_* with "<< message" streaming), so that
// those test programs can be compiled unchanged against this repository's
// drop-in operator API and run where GoogleTest is not installed. Test
// infrastructure only; main() is in ref_gtest/gtest_main.cpp.
//
// Semantics follow GoogleTest's documented behaviour: a failed ASSERT_*
// records the failure and returns from the current function; a failed
// EXPECT_* records it and continues; a test passes when it recorded no
// failure. ASSERT_EQ / ASSERT_NE compare with == / != (floats exactly),
// ASSERT_NEAR with |a - b| <= tol in double.
#pragma once

#include <cmath>
#include <cstdio>
#include <sstream>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

namespace ref_gtest
{
struct TestCase
{
    const char *suite;
    const char *name;
    void (*fn)();
};

inline std::vector<TestCase> &registry()
{
    static std::vector<TestCase> cases;
    return cases;
}

inline int &failures_in_current_test()
{
    static int n = 0;
    return n;
}

struct Registrar
{
    Registrar(const char *suite, const char *name, void (*fn)()) { registry().push_back({suite, name, fn}); }
};

template <typename T, typename = void>
struct Streamable : std::false_type
{
};
template <typename T>
struct Streamable<T, std::void_t<decltype(std::declval<std::ostream &>() << std::declval<const T &>())>>
    : std::true_type
{
};

template <typename T>
std::string show(const T &v)
{
    if constexpr (std::is_same_v<T, unsigned char> || std::is_same_v<T, signed char> || std::is_same_v<T, char>)
        return std::to_string(static_cast<int>(v));
    else if constexpr (std::is_enum_v<T>)
        return std::to_string(static_cast<long long>(v));
    else if constexpr (Streamable<T>::value)
    {
        std::ostringstream os;
        os.precision(9);
        os << v;
        return os.str();
    }
    else
        return "(value)";
}

struct Message
{
    std::ostringstream os;
    Message() = default;
    Message(const Message &o) { os << o.os.str(); }
    template <typename V>
    Message &operator<<(const V &v)
    {
        if constexpr (Streamable<V>::value)
            os << v;
        return *this;
    }
};

// `Failure(...) = Message() << ...` records one failure with its message; the
// assignment returns void so that `return Failure(...) = ...;` is valid in a
// void function (the ASSERT_* form).
struct Failure
{
    const char *file;
    int line;
    std::string what;
    void operator=(const Message &m) const
    {
        ++failures_in_current_test();
        std::string extra = m.os.str();
        std::printf("%s:%d: Failure\n%s\n%s%s", file, line, what.c_str(), extra.c_str(), extra.empty() ? "" : "\n");
    }
};

template <typename A, typename B>
std::string cmp_text(const char *op, const char *ta, const char *tb, const A &a, const B &b)
{
    return std::string("Expected: (") + ta + ") " + op + " (" + tb + "), actual: " + show(a) + " vs " + show(b);
}

inline std::string near_text(const char *ta, const char *tb, const char *tt, double a, double b, double tol)
{
    std::ostringstream os;
    os.precision(9);
    os << "The difference between " << ta << " and " << tb << " is " << std::fabs(a - b) << ", which exceeds "
       << tt << ", where " << ta << " evaluates to " << a << ", " << tb << " evaluates to " << b << ", and " << tt
       << " evaluates to " << tol << ".";
    return os.str();
}
} // namespace ref_gtest

#define TEST(suite, name)                                                                                      \
    static void ref_gtest_body_##suite##_##name();                                                             \
    static ::ref_gtest::Registrar ref_gtest_reg_##suite##_##name(#suite, #name, &ref_gtest_body_##suite##_##name); \
    static void ref_gtest_body_##suite##_##name()

#define REF_GTEST_CHECK_(cond, text, on_fail) \
    if (cond)                                 \
        ;                                     \
    else                                      \
        on_fail ::ref_gtest::Failure{__FILE__, __LINE__, (text)} = ::ref_gtest::Message()

#define REF_GTEST_CMP_(a, b, op, on_fail)                                                              \
    if (auto &&ref_gtest_a_ = (a); true)                                                               \
        if (auto &&ref_gtest_b_ = (b); ref_gtest_a_ op ref_gtest_b_)                                   \
            ;                                                                                          \
        else                                                                                           \
            on_fail ::ref_gtest::Failure{__FILE__, __LINE__,                                           \
                                         ::ref_gtest::cmp_text(#op, #a, #b, ref_gtest_a_, ref_gtest_b_)} = \
                ::ref_gtest::Message()

#define REF_GTEST_NEAR_(a, b, tol, on_fail)                                                                     \
    if (double ref_gtest_a_ = static_cast<double>(a), ref_gtest_b_ = static_cast<double>(b),                    \
        ref_gtest_t_ = static_cast<double>(tol);                                                                \
        std::fabs(ref_gtest_a_ - ref_gtest_b_) <= ref_gtest_t_)                                                 \
        ;                                                                                                       \
    else                                                                                                        \
        on_fail ::ref_gtest::Failure{__FILE__, __LINE__,                                                        \
                                     ::ref_gtest::near_text(#a, #b, #tol, ref_gtest_a_, ref_gtest_b_, ref_gtest_t_)} = \
            ::ref_gtest::Message()

#define ASSERT_EQ(a, b) REF_GTEST_CMP_(a, b, ==, return)
#define ASSERT_NE(a, b) REF_GTEST_CMP_(a, b, !=, return)
#define ASSERT_LT(a, b) REF_GTEST_CMP_(a, b, <, return)
#define ASSERT_LE(a, b) REF_GTEST_CMP_(a, b, <=, return)
#define ASSERT_GT(a, b) REF_GTEST_CMP_(a, b, >, return)
#define ASSERT_GE(a, b) REF_GTEST_CMP_(a, b, >=, return)
#define ASSERT_TRUE(c) REF_GTEST_CHECK_(static_cast<bool>(c), std::string("Value of: ") + #c + "\n  Actual: false", return)
#define ASSERT_FALSE(c) REF_GTEST_CHECK_(!static_cast<bool>(c), std::string("Value of: ") + #c + "\n  Actual: true", return)
#define ASSERT_NEAR(a, b, tol) REF_GTEST_NEAR_(a, b, tol, return)
#define ASSERT_FLOAT_EQ(a, b) ASSERT_EQ(a, b)

#define EXPECT_EQ(a, b) REF_GTEST_CMP_(a, b, ==, )
#define EXPECT_NE(a, b) REF_GTEST_CMP_(a, b, !=, )
#define EXPECT_LT(a, b) REF_GTEST_CMP_(a, b, <, )
#define EXPECT_LE(a, b) REF_GTEST_CMP_(a, b, <=, )
#define EXPECT_GT(a, b) REF_GTEST_CMP_(a, b, >, )
#define EXPECT_GE(a, b) REF_GTEST_CMP_(a, b, >=, )
#define EXPECT_TRUE(c) REF_GTEST_CHECK_(static_cast<bool>(c), std::string("Value of: ") + #c + "\n  Actual: false", )
#define EXPECT_FALSE(c) REF_GTEST_CHECK_(!static_cast<bool>(c), std::string("Value of: ") + #c + "\n  Actual: true", )
#define EXPECT_NEAR(a, b, tol) REF_GTEST_NEAR_(a, b, tol, )
