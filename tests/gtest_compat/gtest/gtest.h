// A minimal GoogleTest-compatible harness: the subset of the gtest interface
// that tinytrain's own unit tests use (TEST, EXPECT_/ASSERT_ comparisons with
// streamed messages, EXPECT_NEAR, EXPECT_FLOAT_EQ, EXPECT_THROW), so those
// test files compile unchanged in an image without GoogleTest. main() is in
// gtest_main.cpp. Test infrastructure only.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

namespace ttgt {

struct Case {
    const char* suite;
    const char* name;
    void (*fn)();
};

inline std::vector<Case>& registry() {
    static std::vector<Case> r;
    return r;
}

inline int& current_failures() {
    static int n = 0;
    return n;
}

struct Registrar {
    Registrar(const char* suite, const char* name, void (*fn)()) {
        registry().push_back({suite, name, fn});
    }
};

// Collects the failure text (and anything streamed after the macro) and
// prints it when the full expression ends.
class Failure {
public:
    Failure(const char* file, int line, const std::string& what) {
        os_ << file << ":" << line << ": Failure\n" << what;
        ++current_failures();
    }
    Failure(const Failure&) = delete;
    ~Failure() { std::cout << os_.str() << std::endl; }
    template <class T>
    Failure& operator<<(const T& v) {
        os_ << v;
        return *this;
    }

private:
    std::ostringstream os_;
};

// `return Returner() = Failure(...) << ...;` ends the test function (ASSERT_*).
struct Returner {
    void operator=(const Failure&) const {}
};

template <class T>
std::string show(const T& v) {
    if constexpr (requires(std::ostream& o, const T& x) { o << x; }) {
        std::ostringstream os;
        os << v;
        return os.str();
    } else {
        return "<unprintable>";
    }
}

template <class A, class B>
std::string binary_text(const char* op, const char* ea, const char* eb, const A& a, const B& b) {
    return std::string("Expected: (") + ea + ") " + op + " (" + eb + "), actual: " + show(a) +
           " vs " + show(b) + "\n";
}

// Float equality within 4 units in the last place (gtest's EXPECT_FLOAT_EQ
// rule): sign-magnitude bit patterns mapped onto one monotonic integer line.
inline bool float_eq(float a, float b) {
    if (std::isnan(a) || std::isnan(b))
        return false;
    auto line = [](float f) {
        uint32_t u;
        std::memcpy(&u, &f, 4);
        return (u & 0x80000000u) ? -static_cast<int64_t>(u & 0x7fffffffu)
                                 : static_cast<int64_t>(u);
    };
    const int64_t d = line(a) - line(b);
    return (d < 0 ? -d : d) <= 4;
}

}  // namespace ttgt

#define TEST(suite, name)                                                            \
    static void ttgt_##suite##_##name();                                             \
    static ::ttgt::Registrar ttgt_reg_##suite##_##name(#suite, #name,                \
                                                       &ttgt_##suite##_##name);      \
    static void ttgt_##suite##_##name()

#define TTGT_CHECK_(cond, text) \
    if (cond)                   \
        ;                       \
    else                        \
        ::ttgt::Failure(__FILE__, __LINE__, text)
#define TTGT_REQUIRE_(cond, text) \
    if (cond)                     \
        ;                         \
    else                          \
        return ::ttgt::Returner() = ::ttgt::Failure(__FILE__, __LINE__, text)

#define TTGT_BIN_(kind, op, a, b) \
    kind(((a)op(b)), ::ttgt::binary_text(#op, #a, #b, (a), (b)))

#define EXPECT_TRUE(c) TTGT_CHECK_(static_cast<bool>(c), "Value of: " #c "\n  Expected: true\n")
#define EXPECT_FALSE(c) TTGT_CHECK_(!static_cast<bool>(c), "Value of: " #c "\n  Expected: false\n")
#define ASSERT_TRUE(c) TTGT_REQUIRE_(static_cast<bool>(c), "Value of: " #c "\n  Expected: true\n")
#define ASSERT_FALSE(c) TTGT_REQUIRE_(!static_cast<bool>(c), "Value of: " #c "\n  Expected: false\n")

#define EXPECT_EQ(a, b) TTGT_BIN_(TTGT_CHECK_, ==, a, b)
#define EXPECT_NE(a, b) TTGT_BIN_(TTGT_CHECK_, !=, a, b)
#define EXPECT_LE(a, b) TTGT_BIN_(TTGT_CHECK_, <=, a, b)
#define EXPECT_LT(a, b) TTGT_BIN_(TTGT_CHECK_, <, a, b)
#define EXPECT_GE(a, b) TTGT_BIN_(TTGT_CHECK_, >=, a, b)
#define EXPECT_GT(a, b) TTGT_BIN_(TTGT_CHECK_, >, a, b)
#define ASSERT_EQ(a, b) TTGT_BIN_(TTGT_REQUIRE_, ==, a, b)
#define ASSERT_NE(a, b) TTGT_BIN_(TTGT_REQUIRE_, !=, a, b)
#define ASSERT_LE(a, b) TTGT_BIN_(TTGT_REQUIRE_, <=, a, b)

#define EXPECT_NEAR(a, b, tol)                                                          \
    TTGT_CHECK_(std::fabs(static_cast<double>(a) - static_cast<double>(b)) <=           \
                    static_cast<double>(tol),                                           \
                std::string("Expected |" #a " - " #b "| <= " #tol ", actual: ") +       \
                    ::ttgt::show(a) + " vs " + ::ttgt::show(b) + "\n")
#define EXPECT_FLOAT_EQ(a, b)                                                           \
    TTGT_CHECK_(::ttgt::float_eq(static_cast<float>(a), static_cast<float>(b)),         \
                std::string("Expected float equality of " #a " and " #b ", actual: ") + \
                    ::ttgt::show(a) + " vs " + ::ttgt::show(b) + "\n")

#define EXPECT_THROW(stmt, exc)                                                    \
    do {                                                                           \
        int ttgt_state_ = 0;                                                       \
        try {                                                                      \
            stmt;                                                                  \
        } catch (const exc&) {                                                     \
            ttgt_state_ = 1;                                                       \
        } catch (...) {                                                            \
            ttgt_state_ = 2;                                                       \
        }                                                                          \
        TTGT_CHECK_(ttgt_state_ == 1, ttgt_state_ == 0                             \
                                          ? "Expected: " #stmt " throws " #exc     \
                                            ".\n  Actual: it throws nothing.\n"    \
                                          : "Expected: " #stmt " throws " #exc     \
                                            ".\n  Actual: it throws another type.\n"); \
    } while (0)
