// gtest/gtest.h -- a minimal googletest-compatible harness (TEST INFRASTRUCTURE
// ONLY), enough to build and run the reference's unit tests against the
// device Network without googletest being installed: TEST, the EXPECT_* and
// ASSERT_* comparisons those tests use (EQ/NE/LT/LE/GT/GE, TRUE/FALSE,
// FLOAT_EQ/DOUBLE_EQ within 4 units in the last place, STREQ), a registry of
// every TEST across translation units and a main() that runs them in
// registration order, printing googletest-style [ RUN ] / [ OK ] /
// [ FAILED ] lines and exiting 1 when any test failed.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <sstream>
#include <string>
#include <type_traits>
#include <vector>

namespace testing {

struct TestInfo {
  const char *suite;
  const char *name;
  void (*body)();
};

inline std::vector<TestInfo> &Registry() {
  static std::vector<TestInfo> r;
  return r;
}

struct Registrar {
  Registrar(const char *suite, const char *name, void (*body)()) {
    Registry().push_back({suite, name, body});
  }
};

namespace internal {

inline bool &Failed() {
  static bool f = false;
  return f;
}

struct AssertionAbort {};  // thrown by ASSERT_* to leave the test body

template <class T, class = void> struct Printable : std::false_type {};
template <class T>
struct Printable<T, std::void_t<decltype(std::declval<std::ostream &>() << std::declval<T>())>>
    : std::true_type {};

template <class T> std::string Show(const T &v) {
  std::ostringstream os;
  if constexpr (std::is_same_v<T, bool>) os << (v ? "true" : "false");
  else if constexpr (std::is_same_v<T, char> || std::is_same_v<T, signed char> ||
                     std::is_same_v<T, unsigned char>)
    os << (int)v;
  else if constexpr (std::is_enum_v<T>) os << (long long)v;
  else if constexpr (Printable<T>::value) {
    os.precision(9);
    os << v;
  } else
    os << "<" << sizeof(T) << "-byte value>";
  return os.str();
}

inline void Report(const char *file, int line, const std::string &what) {
  std::printf("%s:%d: Failure\n%s\n", file, line, what.c_str());
  Failed() = true;
}

// Within 4 units in the last place (googletest's float comparison).
template <class F, class U> bool AlmostEqual(F a, F b) {
  if (std::isnan(a) || std::isnan(b)) return false;
  U ua, ub;
  std::memcpy(&ua, &a, sizeof(F));
  std::memcpy(&ub, &b, sizeof(F));
  constexpr U sign = U(1) << (sizeof(U) * 8 - 1);
  auto biased = [](U u) { return (u & sign) ? ~u + 1 : u | sign; };  // sign-magnitude -> biased
  const U x = biased(ua), y = biased(ub);
  return (x > y ? x - y : y - x) <= 4;
}

}  // namespace internal

inline void InitGoogleTest(int *, char **) {}
inline void InitGoogleTest() {}

inline int RunAllTests() {
  int failed = 0, passed = 0;
  std::vector<std::string> failures;
  const auto &tests = Registry();
  std::printf("[==========] Running %zu tests.\n", tests.size());
  for (const auto &t : tests) {
    std::printf("[ RUN      ] %s.%s\n", t.suite, t.name);
    std::fflush(stdout);
    internal::Failed() = false;
    try {
      t.body();
    } catch (const internal::AssertionAbort &) {
    } catch (const std::exception &e) {
      internal::Report("(test body)", 0, std::string("uncaught exception: ") + e.what());
    }
    if (internal::Failed()) {
      ++failed;
      failures.push_back(std::string(t.suite) + "." + t.name);
      std::printf("[  FAILED  ] %s.%s\n", t.suite, t.name);
    } else {
      ++passed;
      std::printf("[       OK ] %s.%s\n", t.suite, t.name);
    }
    std::fflush(stdout);
  }
  std::printf("[==========] %zu tests ran.\n[  PASSED  ] %d tests.\n", tests.size(), passed);
  if (failed) {
    std::printf("[  FAILED  ] %d tests, listed below:\n", failed);
    for (const auto &f : failures) std::printf("[  FAILED  ] %s\n", f.c_str());
  }
  return failed ? 1 : 0;
}

}  // namespace testing

#define RUN_ALL_TESTS() ::testing::RunAllTests()

#define TEST(Suite, Name)                                                                 \
  static void Suite##_##Name##_TestBody();                                               \
  static ::testing::Registrar Suite##_##Name##_Registrar(#Suite, #Name,                  \
                                                         &Suite##_##Name##_TestBody);    \
  static void Suite##_##Name##_TestBody()

#define GTEST_CMP_(a, b, op, fatal)                                                       \
  do {                                                                                    \
    const auto &gt_a_ = (a);                                                             \
    const auto &gt_b_ = (b);                                                             \
    if (!(gt_a_ op gt_b_)) {                                                              \
      ::testing::internal::Report(__FILE__, __LINE__,                                     \
                                  "Expected: (" #a ") " #op " (" #b "), actual: " +       \
                                      ::testing::internal::Show(gt_a_) + " vs " +         \
                                      ::testing::internal::Show(gt_b_));                  \
      if (fatal) throw ::testing::internal::AssertionAbort{};                             \
    }                                                                                     \
  } while (0)

#define GTEST_BOOL_(c, want, fatal)                                                       \
  do {                                                                                    \
    if (static_cast<bool>(c) != (want)) {                                                 \
      ::testing::internal::Report(__FILE__, __LINE__,                                     \
                                  "Value of: " #c "\n  Expected: " #want);                \
      if (fatal) throw ::testing::internal::AssertionAbort{};                             \
    }                                                                                     \
  } while (0)

#define GTEST_FP_(a, b, F, U, fatal)                                                      \
  do {                                                                                    \
    const F gt_a_ = static_cast<F>(a), gt_b_ = static_cast<F>(b);                         \
    if (!::testing::internal::AlmostEqual<F, U>(gt_a_, gt_b_)) {                          \
      ::testing::internal::Report(__FILE__, __LINE__,                                     \
                                  "Expected equality of (" #a ") and (" #b "): " +        \
                                      ::testing::internal::Show(gt_a_) + " vs " +         \
                                      ::testing::internal::Show(gt_b_));                  \
      if (fatal) throw ::testing::internal::AssertionAbort{};                             \
    }                                                                                     \
  } while (0)

#define EXPECT_EQ(a, b) GTEST_CMP_(a, b, ==, false)
#define EXPECT_NE(a, b) GTEST_CMP_(a, b, !=, false)
#define EXPECT_LT(a, b) GTEST_CMP_(a, b, <, false)
#define EXPECT_LE(a, b) GTEST_CMP_(a, b, <=, false)
#define EXPECT_GT(a, b) GTEST_CMP_(a, b, >, false)
#define EXPECT_GE(a, b) GTEST_CMP_(a, b, >=, false)
#define ASSERT_EQ(a, b) GTEST_CMP_(a, b, ==, true)
#define ASSERT_NE(a, b) GTEST_CMP_(a, b, !=, true)
#define ASSERT_LT(a, b) GTEST_CMP_(a, b, <, true)
#define ASSERT_LE(a, b) GTEST_CMP_(a, b, <=, true)
#define ASSERT_GT(a, b) GTEST_CMP_(a, b, >, true)
#define ASSERT_GE(a, b) GTEST_CMP_(a, b, >=, true)
#define EXPECT_TRUE(c) GTEST_BOOL_(c, true, false)
#define EXPECT_FALSE(c) GTEST_BOOL_(c, false, false)
#define ASSERT_TRUE(c) GTEST_BOOL_(c, true, true)
#define ASSERT_FALSE(c) GTEST_BOOL_(c, false, true)
#define EXPECT_FLOAT_EQ(a, b) GTEST_FP_(a, b, float, uint32_t, false)
#define EXPECT_DOUBLE_EQ(a, b) GTEST_FP_(a, b, double, uint64_t, false)
#define ASSERT_FLOAT_EQ(a, b) GTEST_FP_(a, b, float, uint32_t, true)
#define ASSERT_DOUBLE_EQ(a, b) GTEST_FP_(a, b, double, uint64_t, true)
#define EXPECT_STREQ(a, b)                                                                \
  do {                                                                                    \
    const char *gt_a_ = (a), *gt_b_ = (b);                                                \
    if (!(gt_a_ && gt_b_ ? std::strcmp(gt_a_, gt_b_) == 0 : gt_a_ == gt_b_))              \
      ::testing::internal::Report(__FILE__, __LINE__,                                     \
                                  std::string("Expected equal strings: ") +               \
                                      (gt_a_ ? gt_a_ : "(null)") + " vs " +               \
                                      (gt_b_ ? gt_b_ : "(null)"));                        \
  } while (0)
