// Minimal stand-in for <gtest/gtest.h> used only to compile the reference's
// golden-attention test file as a library (oracle/_ref).  TEST bodies become
// uninstantiated templates, so none of them is compiled into code or run; the
// file's static helpers (random_floats, cpu_attention) stay callable.
#pragma once

namespace vk_gtest_shim {
struct Sink {
    template <class T>
    Sink& operator<<(const T&) { return *this; }
};
}  // namespace vk_gtest_shim

#define TEST(suite, name) template <int VkShimUnused> void vk_shim_##suite##_##name()
#define VK_SHIM_SINK ::vk_gtest_shim::Sink()
#define EXPECT_TRUE(a) VK_SHIM_SINK
#define EXPECT_FALSE(a) VK_SHIM_SINK
#define EXPECT_EQ(a, b) VK_SHIM_SINK
#define EXPECT_NE(a, b) VK_SHIM_SINK
#define EXPECT_LT(a, b) VK_SHIM_SINK
#define EXPECT_LE(a, b) VK_SHIM_SINK
#define EXPECT_GT(a, b) VK_SHIM_SINK
#define EXPECT_GE(a, b) VK_SHIM_SINK
#define EXPECT_NEAR(a, b, t) VK_SHIM_SINK
#define EXPECT_FLOAT_EQ(a, b) VK_SHIM_SINK
#define ASSERT_TRUE(a) VK_SHIM_SINK
#define ASSERT_EQ(a, b) VK_SHIM_SINK
#define ASSERT_NE(a, b) VK_SHIM_SINK
