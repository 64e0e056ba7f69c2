// Minimal stand-in for <gtest/gtest.h>, just enough for the reference's test files to
// compile as libraries (GoogleTest is not installed here). Test bodies compile into
// member functions nobody calls; only the files' helper functions are used.
#pragma once
#include <ostream>
namespace testing {
class Test {
public:
    virtual ~Test() {}
protected:
    virtual void SetUp() {}
    virtual void TearDown() {}
};
}  // namespace testing
struct B2GtestNullStream {
    template <class T> B2GtestNullStream& operator<<(const T&) { return *this; }
};
#define B2_GTEST_SINK if (true) {} else B2GtestNullStream()
#define EXPECT_LT(a, b) B2_GTEST_SINK
#define EXPECT_LE(a, b) B2_GTEST_SINK
#define EXPECT_GT(a, b) B2_GTEST_SINK
#define EXPECT_EQ(a, b) B2_GTEST_SINK
#define EXPECT_NEAR(a, b, c) B2_GTEST_SINK
#define EXPECT_TRUE(a) B2_GTEST_SINK
#define ASSERT_LT(a, b) B2_GTEST_SINK
#define ASSERT_EQ(a, b) B2_GTEST_SINK
#define ASSERT_TRUE(a) B2_GTEST_SINK
#define TEST_F(F, N)                                \
    class F##_##N##_Test : public F {               \
    public:                                         \
        void TestBody();                            \
    };                                              \
    void F##_##N##_Test::TestBody()
