# Builds the reference harness's OWN test suites and flash-attention bench, unchanged, against the
# B200 library: the sources are compiled where they lie in the reference tree, with
#   * ascend-npu-harness_b200/host/reference_runners ahead of ops/<op>/runner on the include path
#     (the runner seam, run on the GPU) and runner_bridge.cpp in place of the runner .cpp files,
#   * the reference's harness core (src/accuracy, dtype, shape, test_utils) except
#     src/ascend_runtime.cpp, whose role libhc_harness.so's device runtime takes,
#   * tests/cpp/gtest_shim in place of GoogleTest (not installed here).
# Outputs (test infrastructure, git-ignored): _bin/reference/test_<op>, _bin/reference/bench_<op>.
#
# Usage: make -f tests/cpp/reference_suite.mk REF=<reference tree>   (or HC_REFERENCE_DIR=<tree>)
# Needs ascend-npu-harness_b200/lib/libhc_harness.so + libhc_b200.so (build.py).
REF ?= $(HC_REFERENCE_DIR)
CXX ?= g++
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
ROOT := $(abspath $(HERE)../..)
LIB := $(ROOT)/ascend-npu-harness_b200/lib
BRIDGE := $(ROOT)/ascend-npu-harness_b200/host/reference_runners
OUT := $(HERE)_bin/reference
OBJ := $(OUT)/obj

OPS := elementwise_add axpy_scalar_affine broadcast_binary activation_gelu_silu reduce_sum_lastdim \
       transpose_2d_4d layer_norm rms_norm_rope_fused matmul_bias flash_attention_fwd_fused
BENCHES := flash_attention_fwd_fused layer_norm elementwise_add

ifeq ($(strip $(REF)),)
all:
	@echo "reference tree not given (REF=... or HC_REFERENCE_DIR): nothing to build"
else ifeq ($(wildcard $(REF)/tests/test_harness_core.cpp),)
all:
	@echo "reference tree $(REF) not present: keeping any prebuilt binaries"
else

# Flags follow the reference's Release preset (cmake/CompilerOptions.cmake: -O3 -DNDEBUG, C++17).
OP_INCS = $(foreach o,$(OPS),$(foreach s,golden host,-I$(REF)/ops/$(o)/$(s)))
RUNNER_INCS = $(foreach o,$(OPS),-I$(REF)/ops/$(o)/runner)
CXXFLAGS := -O3 -DNDEBUG -std=gnu++17 -DHARNESS_HAS_GTEST=1 -DHARNESS_HAS_CUDA=1 \
            -I$(HERE)gtest_shim -I$(BRIDGE) -I$(ROOT)/ascend-npu-harness_b200/host/include -I$(ROOT)/include \
            -I$(REF)/include $(OP_INCS) $(RUNNER_INCS)
LDFLAGS := -L$(LIB) -lhc_harness -lhc_b200 -Wl,-rpath,$(LIB) -lpthread

CORE_SRCS := $(REF)/src/accuracy.cpp $(REF)/src/dtype.cpp $(REF)/src/shape.cpp $(REF)/src/test_utils.cpp
CORE_OBJS := $(patsubst $(REF)/src/%.cpp,$(OBJ)/core_%.o,$(CORE_SRCS))
GOLDEN_SRCS := $(foreach o,$(OPS),$(wildcard $(REF)/ops/$(o)/golden/*.cpp))
TILING_SRCS := $(foreach o,$(OPS),$(wildcard $(REF)/ops/$(o)/host/*.cpp))
OP_OBJS := $(foreach f,$(GOLDEN_SRCS) $(TILING_SRCS),$(OBJ)/$(subst /,_,$(patsubst $(REF)/ops/%.cpp,%,$(f))).o)
BRIDGE_OBJ := $(OBJ)/runner_bridge.o
LIB_OBJS := $(CORE_OBJS) $(OP_OBJS) $(BRIDGE_OBJ)

TESTS := $(OUT)/test_harness_core $(foreach o,$(OPS),$(OUT)/test_$(o))
BENCH_BINS := $(foreach o,$(BENCHES),$(OUT)/bench_$(o))

all: $(TESTS) $(BENCH_BINS)

$(OBJ)/core_%.o: $(REF)/src/%.cpp
	@mkdir -p $(OBJ)
	$(CXX) $(CXXFLAGS) -c $< -o $@

define op_obj_rule
$(OBJ)/$(subst /,_,$(patsubst $(REF)/ops/%.cpp,%,$(1))).o: $(1)
	@mkdir -p $(OBJ)
	$(CXX) $(CXXFLAGS) -c $(1) -o $$@
endef
$(foreach f,$(GOLDEN_SRCS) $(TILING_SRCS),$(eval $(call op_obj_rule,$(f))))

$(BRIDGE_OBJ): $(BRIDGE)/runner_bridge.cpp $(wildcard $(BRIDGE)/*.hpp)
	@mkdir -p $(OBJ)
	$(CXX) $(CXXFLAGS) -c $< -o $@

# gtest_main's main() comes from the shim header, defined in the test's own translation unit.
$(OUT)/test_%: $(REF)/tests/test_%.cpp $(LIB_OBJS) $(wildcard $(BRIDGE)/*.hpp) $(HERE)mini_gtest.hpp $(LIB)/libhc_harness.so
	$(CXX) $(CXXFLAGS) -DHC_GTEST_SHIM_MAIN $< $(LIB_OBJS) -o $@ $(LDFLAGS)

define bench_rule
$(OUT)/bench_$(1): $(REF)/ops/$(1)/bench/bench_$(1).cpp $(LIB_OBJS) $(wildcard $(BRIDGE)/*.hpp) $(LIB)/libhc_harness.so
	$(CXX) $(CXXFLAGS) $$< $(LIB_OBJS) -o $$@ $(LDFLAGS)
endef
$(foreach o,$(BENCHES),$(eval $(call bench_rule,$(o))))

endif

clean:
	rm -rf $(OUT)

.PHONY: all clean
