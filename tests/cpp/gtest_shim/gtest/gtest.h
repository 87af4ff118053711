// Stand-in for <gtest/gtest.h> (GoogleTest is not installed here): the reference harness's test
// files include it unchanged and get the GoogleTest-compatible subset of mini_gtest.hpp, with
// gtest_main's main() (MINI_GTEST_MAIN) defined in the translation unit that sets
// HC_GTEST_SHIM_MAIN.
#pragma once
#include "../../mini_gtest.hpp"
#ifdef HC_GTEST_SHIM_MAIN
MINI_GTEST_MAIN
#endif
