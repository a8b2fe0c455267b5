// main() of the reference unit-test binary built against the minimal
// googletest-compatible harness (TEST INFRASTRUCTURE ONLY).
#include <gtest/gtest.h>

int main(int argc, char **argv) {
  ::testing::InitGoogleTest(&argc, argv);
  return RUN_ALL_TESTS();
}
