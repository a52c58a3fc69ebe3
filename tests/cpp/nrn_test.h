// nrn_test.h -- a minimal test harness for the C++ API tests (the reference
// uses GoogleTest, which this image does not have; the assertions below
// keep its names and meaning).
#pragma once

#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

namespace nrn_test {

struct Case {
    const char* suite;
    const char* name;
    std::function<void()> fn;
};

inline std::vector<Case>& registry() {
    static std::vector<Case> r;
    return r;
}

inline int& failures() {
    static int f = 0;
    return f;
}

struct Registrar {
    Registrar(const char* s, const char* n, std::function<void()> f) { registry().push_back({s, n, std::move(f)}); }
};

inline void report(const char* file, int line, const std::string& what) {
    std::printf("  FAIL %s:%d: %s\n", file, line, what.c_str());
    ++failures();
}

}  // namespace nrn_test

#define TEST(suite, name)                                                                   \
    static void suite##_##name##_body();                                                    \
    static nrn_test::Registrar suite##_##name##_reg(#suite, #name, suite##_##name##_body); \
    static void suite##_##name##_body()

#define NRN_EXPECT_IMPL(cond, text)                                         \
    do {                                                                    \
        if (!(cond)) nrn_test::report(__FILE__, __LINE__, text);            \
    } while (0)

#define EXPECT_TRUE(c) NRN_EXPECT_IMPL((c), "EXPECT_TRUE(" #c ")")
#define EXPECT_FALSE(c) NRN_EXPECT_IMPL(!(c), "EXPECT_FALSE(" #c ")")
#define EXPECT_EQ(a, b) NRN_EXPECT_IMPL((a) == (b), "EXPECT_EQ(" #a ", " #b ")")
#define EXPECT_NE(a, b) NRN_EXPECT_IMPL((a) != (b), "EXPECT_NE(" #a ", " #b ")")
#define EXPECT_GT(a, b) NRN_EXPECT_IMPL((a) > (b), "EXPECT_GT(" #a ", " #b ")")
#define EXPECT_GE(a, b) NRN_EXPECT_IMPL((a) >= (b), "EXPECT_GE(" #a ", " #b ")")
#define EXPECT_LT(a, b) NRN_EXPECT_IMPL((a) < (b), "EXPECT_LT(" #a ", " #b ")")
#define EXPECT_LE(a, b) NRN_EXPECT_IMPL((a) <= (b), "EXPECT_LE(" #a ", " #b ")")
#define EXPECT_NEAR(a, b, tol) NRN_EXPECT_IMPL(std::fabs((double)(a) - (double)(b)) <= (tol), "EXPECT_NEAR(" #a ", " #b ")")
#define EXPECT_DOUBLE_EQ(a, b) NRN_EXPECT_IMPL((double)(a) == (double)(b), "EXPECT_DOUBLE_EQ(" #a ", " #b ")")
#define EXPECT_FLOAT_EQ(a, b) NRN_EXPECT_IMPL((float)(a) == (float)(b), "EXPECT_FLOAT_EQ(" #a ", " #b ")")
#define EXPECT_THROW(stmt, Exc)                                         \
    do {                                                                \
        bool caught_ = false;                                           \
        try { stmt; } catch (const Exc&) { caught_ = true; } catch (...) {} \
        NRN_EXPECT_IMPL(caught_, "EXPECT_THROW(" #stmt ", " #Exc ")");  \
    } while (0)
#define EXPECT_NO_THROW(stmt)                                           \
    do {                                                                \
        bool ok_ = true;                                                \
        try { stmt; } catch (...) { ok_ = false; }                      \
        NRN_EXPECT_IMPL(ok_, "EXPECT_NO_THROW(" #stmt ")");             \
    } while (0)
#define ASSERT_TRUE(c) do { if (!(c)) { nrn_test::report(__FILE__, __LINE__, "ASSERT_TRUE(" #c ")"); return; } } while (0)
#define SUCCEED() (void)0

// main(): runs every registered test (or those whose "Suite.Name" contains
// argv[1]); exit status 1 on any failure.
#define NRN_TEST_MAIN()                                                                       \
    int main(int argc, char** argv) {                                                         \
        int ran = 0;                                                                          \
        for (auto& c : nrn_test::registry()) {                                                \
            std::string full = std::string(c.suite) + "." + c.name;                            \
            if (argc > 1 && full.find(argv[1]) == std::string::npos) continue;                \
            const int before = nrn_test::failures();                                          \
            try {                                                                             \
                c.fn();                                                                       \
            } catch (const std::exception& e) {                                               \
                nrn_test::report(c.suite, 0, std::string("exception: ") + e.what());          \
            }                                                                                 \
            std::printf("[%s] %s\n", nrn_test::failures() == before ? "  OK  " : " FAIL ", full.c_str()); \
            ++ran;                                                                            \
        }                                                                                     \
        std::printf("%d tests, %d failures\n", ran, nrn_test::failures());                    \
        return nrn_test::failures() == 0 && ran > 0 ? 0 : 1;                                  \
    }
