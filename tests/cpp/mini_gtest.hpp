// A small GoogleTest-compatible test framework (own code; GoogleTest is not installed here).
//
// Supports the subset the harness's C++ tests use: TEST, TEST_F (fixtures with SetUp/TearDown),
// value-parameterized suites (TestWithParam<T>, GetParam(), TEST_P, INSTANTIATE_TEST_SUITE_P with
// ::testing::Values, named "<prefix>/<Suite>.<name>/<index>" as GoogleTest names them),
// EXPECT_/ASSERT_ TRUE, FALSE, EQ, NE, LT, LE, GT, GE, NEAR, FLOAT_EQ, DOUBLE_EQ, THROW,
// NO_THROW, streaming extra context with <<, GTEST_SKIP(), --gtest_filter (':'-separated
// patterns with * and ?, negatives after '-') and --gtest_list_tests.  Output follows GoogleTest's
// "[ RUN      ] / [       OK ] / [  FAILED  ]" lines; the exit status is 1 when a test failed.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <functional>
#include <iostream>
#include <memory>
#include <sstream>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

namespace testing {

class Test {
public:
    virtual ~Test() = default;
    virtual void SetUp() {}
    virtual void TearDown() {}
    virtual void TestBody() = 0;
};

class Message {
public:
    template <class T>
    Message& operator<<(const T& v) {
        ss_ << v;
        return *this;
    }
    std::string str() const { return ss_.str(); }

private:
    std::ostringstream ss_;
};

namespace internal {

struct TestInfo {
    std::string suite, name;
    std::function<Test*()> make;
};

inline std::vector<TestInfo>& registry() {
    static std::vector<TestInfo> r;
    return r;
}

struct State {
    bool failed = false;
    bool skipped = false;
};

inline State& state() {
    static State s;
    return s;
}

inline bool register_test(const char* suite, const char* name, std::function<Test*()> make) {
    registry().push_back({suite, name, std::move(make)});
    return true;
}

// Records a failure; `operator=` takes the streamed message so that `return Helper(...) = Message()
// << ...;` works inside a void test body (the GoogleTest idiom).
class AssertHelper {
public:
    AssertHelper(const char* file, int line, std::string summary) : file_(file), line_(line), summary_(std::move(summary)) {}
    void operator=(const Message& m) const {
        state().failed = true;
        std::cout << file_ << ":" << line_ << ": Failure\n" << summary_;
        const std::string extra = m.str();
        if (!extra.empty()) std::cout << "\n" << extra;
        std::cout << std::endl;
    }

private:
    const char* file_;
    int line_;
    std::string summary_;
};

class SkipHelper {
public:
    SkipHelper(const char* file, int line) : file_(file), line_(line) {}
    void operator=(const Message& m) const {
        state().skipped = true;
        std::cout << file_ << ":" << line_ << ": Skipped\n" << m.str() << std::endl;
    }

private:
    const char* file_;
    int line_;
};

// Prints a value for a failure message: with its operator<< when it has one, as its underlying
// integer for an enum without one, else as "<N-byte object>" (GoogleTest prints bytes).
template <class T, class = void>
struct Streamable : std::false_type {};
template <class T>
struct Streamable<T, decltype(void(std::declval<std::ostream&>() << std::declval<const T&>()))> : std::true_type {};

template <class T>
void print_value(std::ostream& os, const T& v) {
    if constexpr (Streamable<T>::value) {
        os << v;
    } else if constexpr (std::is_enum<T>::value) {
        os << static_cast<long long>(v);
    } else {
        os << "<" << sizeof(T) << "-byte object>";
    }
}

template <class A, class B>
std::string cmp_summary(const char* op, const char* ea, const char* eb, const A& a, const B& b) {
    std::ostringstream ss;
    ss << "Expected: (" << ea << ") " << op << " (" << eb << "), actual: ";
    print_value(ss, a);
    ss << " vs ";
    print_value(ss, b);
    return ss.str();
}

// Equality within 4 units in the last place, as GoogleTest's FLOAT_EQ / DOUBLE_EQ.
template <class F, class U>
bool almost_equal(F a, F b) {
    if (std::isnan(a) || std::isnan(b)) return false;
    U ua, ub;
    std::memcpy(&ua, &a, sizeof(F));
    std::memcpy(&ub, &b, sizeof(F));
    const U sign = U(1) << (sizeof(U) * 8 - 1);
    auto biased = [sign](U u) { return (u & sign) ? ~u + 1 : (u | sign); };
    const U x = biased(ua), y = biased(ub);
    return (x >= y ? x - y : y - x) <= 4;
}

inline bool glob_match(const char* p, const char* s) {
    if (!*p) return !*s;
    if (*p == '*') return glob_match(p + 1, s) || (*s && glob_match(p, s + 1));
    if (*s && (*p == '?' || *p == *s)) return glob_match(p + 1, s + 1);
    return false;
}

inline bool any_match(const std::string& patterns, const std::string& full) {
    size_t start = 0;
    while (start <= patterns.size()) {
        size_t end = patterns.find(':', start);
        if (end == std::string::npos) end = patterns.size();
        const std::string p = patterns.substr(start, end - start);
        if (!p.empty() && glob_match(p.c_str(), full.c_str())) return true;
        start = end + 1;
    }
    return false;
}

inline std::string& filter() {
    static std::string f = "*";
    return f;
}
inline bool& list_only() {
    static bool l = false;
    return l;
}

// ---- value-parameterized tests --------------------------------------------------------------
// TEST_P records a pattern per (suite, name); INSTANTIATE_TEST_SUITE_P records the suite's values.
// The cross product is expanded into ordinary registry entries when the tests are first run, so
// the order of the two macros in a file does not matter.
struct ParamPattern {
    std::string suite, name;
    std::function<Test*()> make;
};

inline std::vector<ParamPattern>& param_patterns() {
    static std::vector<ParamPattern> p;
    return p;
}

inline std::vector<std::function<void()>>& param_expansions() {
    static std::vector<std::function<void()>> e;
    return e;
}

inline bool register_param_pattern(const char* suite, const char* name, std::function<Test*()> make) {
    param_patterns().push_back({suite, name, std::move(make)});
    return true;
}

inline void expand_param_tests() {
    static bool done = false;
    if (done) return;
    done = true;
    for (auto& e : param_expansions()) e();
}

}  // namespace internal

template <class T>
class WithParamInterface {
public:
    using ParamType = T;
    virtual ~WithParamInterface() = default;
    const T& GetParam() const { return *current(); }
    // The value of the test instance being constructed and run (tests run one at a time).
    static const T*& current() {
        static const T* p = nullptr;
        return p;
    }
};

template <class T>
class TestWithParam : public Test, public WithParamInterface<T> {};

template <class T>
struct ValueList {
    std::vector<T> values;
};

template <class T, class... Ts>
ValueList<T> Values(T first, Ts... rest) {
    return ValueList<T>{std::vector<T>{std::move(first), static_cast<T>(std::move(rest))...}};
}

namespace internal {

template <class Fixture, class T>
bool register_instantiation(const char* prefix, const char* suite, ValueList<T> list) {
    using P = typename Fixture::ParamType;
    auto values = std::make_shared<std::vector<P>>();
    for (auto& v : list.values) values->push_back(static_cast<P>(v));
    const std::string pre = prefix, su = suite;
    param_expansions().push_back([values, pre, su] {
        for (const auto& pat : param_patterns()) {
            if (pat.suite != su) continue;
            for (size_t i = 0; i < values->size(); ++i) {
                auto make = pat.make;
                const P* value = &(*values)[i];
                registry().push_back({pre + "/" + su, pat.name + "/" + std::to_string(i), [make, value, values] {
                                          WithParamInterface<P>::current() = value;
                                          return make();
                                      }});
            }
        }
    });
    return true;
}

}  // namespace internal

inline void InitGoogleTest(int* argc, char** argv) {
    for (int i = 1; i < *argc; ++i) {
        const char* a = argv[i];
        if (std::strncmp(a, "--gtest_filter=", 15) == 0) internal::filter() = a + 15;
        if (std::strcmp(a, "--gtest_list_tests") == 0) internal::list_only() = true;
    }
}

inline int RunAllTests() {
    using namespace internal;
    expand_param_tests();
    std::string pos = filter(), neg;
    const size_t dash = pos.find('-');
    if (dash != std::string::npos) {
        neg = pos.substr(dash + 1);
        pos = pos.substr(0, dash);
        if (pos.empty()) pos = "*";
    }
    std::vector<const TestInfo*> sel;
    for (const auto& t : registry()) {
        const std::string full = t.suite + "." + t.name;
        if (any_match(pos, full) && !(neg.size() && any_match(neg, full))) sel.push_back(&t);
    }
    if (list_only()) {
        for (const auto* t : sel) std::cout << t->suite << "." << t->name << "\n";
        return 0;
    }
    std::cout << "[==========] Running " << sel.size() << " tests." << std::endl;
    std::vector<std::string> failed;
    size_t passed = 0, skipped = 0;
    for (const auto* t : sel) {
        const std::string full = t->suite + "." + t->name;
        std::cout << "[ RUN      ] " << full << std::endl;
        state() = State{};
        Test* obj = nullptr;
        try {
            obj = t->make();
            obj->SetUp();
            if (!state().failed && !state().skipped) obj->TestBody();
            obj->TearDown();
        } catch (const std::exception& e) {
            state().failed = true;
            std::cout << "unexpected exception: " << e.what() << std::endl;
        } catch (...) {
            state().failed = true;
            std::cout << "unexpected exception of unknown type" << std::endl;
        }
        delete obj;
        if (state().failed) {
            failed.push_back(full);
            std::cout << "[  FAILED  ] " << full << std::endl;
        } else if (state().skipped) {
            ++skipped;
            std::cout << "[  SKIPPED ] " << full << std::endl;
        } else {
            ++passed;
            std::cout << "[       OK ] " << full << std::endl;
        }
    }
    std::cout << "[==========] " << sel.size() << " tests ran.\n[  PASSED  ] " << passed << " tests." << std::endl;
    if (skipped) std::cout << "[  SKIPPED ] " << skipped << " tests." << std::endl;
    if (!failed.empty()) {
        std::cout << "[  FAILED  ] " << failed.size() << " tests, listed below:" << std::endl;
        for (const auto& f : failed) std::cout << "[  FAILED  ] " << f << std::endl;
        return 1;
    }
    return 0;
}

}  // namespace testing

#define RUN_ALL_TESTS() ::testing::RunAllTests()

#define MGT_CLASS_(suite, name) suite##_##name##_Test

#define MGT_TEST_(suite, name, parent)                                                               \
    class MGT_CLASS_(suite, name) : public parent {                                                  \
    public:                                                                                          \
        void TestBody() override;                                                                    \
    };                                                                                               \
    static const bool suite##_##name##_registered_ = ::testing::internal::register_test(            \
        #suite, #name, [] { return static_cast<::testing::Test*>(new MGT_CLASS_(suite, name)); }); \
    void MGT_CLASS_(suite, name)::TestBody()

#define TEST(suite, name) MGT_TEST_(suite, name, ::testing::Test)

#define TEST_P(fixture, name)                                                                          \
    class MGT_CLASS_(fixture, name) : public fixture {                                                 \
    public:                                                                                            \
        void TestBody() override;                                                                      \
    };                                                                                                 \
    static const bool fixture##_##name##_pattern_ = ::testing::internal::register_param_pattern(      \
        #fixture, #name, [] { return static_cast<::testing::Test*>(new MGT_CLASS_(fixture, name)); }); \
    void MGT_CLASS_(fixture, name)::TestBody()

#define INSTANTIATE_TEST_SUITE_P(prefix, fixture, generator)                                       \
    static const bool prefix##_##fixture##_instantiated_ =                                         \
        ::testing::internal::register_instantiation<fixture>(#prefix, #fixture, generator)
#define TEST_F(fixture, name) MGT_TEST_(fixture, name, fixture)

// on_failure is empty for EXPECT_* (continue) and `return` for ASSERT_* (leave the test body).
#define MGT_CHECK_(cond, summary, on_failure) \
    if (cond)                                 \
        ;                                     \
    else                                      \
        on_failure ::testing::internal::AssertHelper(__FILE__, __LINE__, summary) = ::testing::Message()

#define MGT_BOOL_(expr, want, on_failure) \
    MGT_CHECK_(static_cast<bool>(expr) == want, std::string("Value of: ") + #expr + "\n  Expected: " + (want ? "true" : "false"), on_failure)

#define MGT_CMP_(a, b, op, on_failure) \
    MGT_CHECK_((a)op(b), ::testing::internal::cmp_summary(#op, #a, #b, (a), (b)), on_failure)

#define EXPECT_TRUE(c) MGT_BOOL_(c, true, )
#define EXPECT_FALSE(c) MGT_BOOL_(c, false, )
#define ASSERT_TRUE(c) MGT_BOOL_(c, true, return)
#define ASSERT_FALSE(c) MGT_BOOL_(c, false, return)
#define EXPECT_EQ(a, b) MGT_CMP_(a, b, ==, )
#define EXPECT_NE(a, b) MGT_CMP_(a, b, !=, )
#define EXPECT_LT(a, b) MGT_CMP_(a, b, <, )
#define EXPECT_LE(a, b) MGT_CMP_(a, b, <=, )
#define EXPECT_GT(a, b) MGT_CMP_(a, b, >, )
#define EXPECT_GE(a, b) MGT_CMP_(a, b, >=, )
#define ASSERT_EQ(a, b) MGT_CMP_(a, b, ==, return)
#define ASSERT_NE(a, b) MGT_CMP_(a, b, !=, return)
#define ASSERT_LT(a, b) MGT_CMP_(a, b, <, return)
#define ASSERT_LE(a, b) MGT_CMP_(a, b, <=, return)
#define ASSERT_GT(a, b) MGT_CMP_(a, b, >, return)
#define ASSERT_GE(a, b) MGT_CMP_(a, b, >=, return)

#define MGT_NEAR_(a, b, tol, on_failure)                                                                    \
    MGT_CHECK_(std::fabs(static_cast<double>(a) - static_cast<double>(b)) <= static_cast<double>(tol),     \
               ::testing::internal::cmp_summary("within " #tol " of", #a, #b, (a), (b)), on_failure)
#define EXPECT_NEAR(a, b, tol) MGT_NEAR_(a, b, tol, )
#define ASSERT_NEAR(a, b, tol) MGT_NEAR_(a, b, tol, return)

#define EXPECT_FLOAT_EQ(a, b)                                                                              \
    MGT_CHECK_((::testing::internal::almost_equal<float, uint32_t>(static_cast<float>(a), static_cast<float>(b))), \
               ::testing::internal::cmp_summary("FLOAT_EQ", #a, #b, (a), (b)), )
#define EXPECT_DOUBLE_EQ(a, b)                                                                                \
    MGT_CHECK_((::testing::internal::almost_equal<double, uint64_t>(static_cast<double>(a), static_cast<double>(b))), \
               ::testing::internal::cmp_summary("DOUBLE_EQ", #a, #b, (a), (b)), )

#define MGT_THROW_(stmt, exc, on_failure)                                             \
    MGT_CHECK_(([&]() -> bool {                                                       \
                   try {                                                              \
                       stmt;                                                          \
                   } catch (const exc&) {                                             \
                       return true;                                                   \
                   } catch (...) {                                                    \
                   }                                                                  \
                   return false;                                                      \
               }()),                                                                  \
               std::string("Expected: " #stmt " throws an exception of type " #exc), on_failure)
#define EXPECT_THROW(stmt, exc) MGT_THROW_(stmt, exc, )
#define ASSERT_THROW(stmt, exc) MGT_THROW_(stmt, exc, return)

#define MGT_NO_THROW_(stmt, on_failure)                                     \
    MGT_CHECK_(([&]() -> bool {                                             \
                   try {                                                    \
                       stmt;                                                \
                   } catch (const std::exception& e) {                      \
                       std::cout << "threw: " << e.what() << std::endl;     \
                       return false;                                        \
                   } catch (...) {                                          \
                       return false;                                        \
                   }                                                        \
                   return true;                                             \
               }()),                                                        \
               std::string("Expected: " #stmt " does not throw"), on_failure)
#define EXPECT_NO_THROW(stmt) MGT_NO_THROW_(stmt, )
#define ASSERT_NO_THROW(stmt) MGT_NO_THROW_(stmt, return)

#define GTEST_SKIP() return ::testing::internal::SkipHelper(__FILE__, __LINE__) = ::testing::Message()

#define MINI_GTEST_MAIN                                  \
    int main(int argc, char** argv) {                    \
        ::testing::InitGoogleTest(&argc, argv);          \
        return RUN_ALL_TESTS();                          \
    }
