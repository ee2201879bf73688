# Builds the interposer (libnccl_b200.so: C++ runtime + sm_100a kernels) and
# the CUDA-free core library (libnb_core.so) used by the CPU test-suite.
CUDA ?= /usr/local/cuda
NVCC ?= $(CUDA)/bin/nvcc
CXX ?= g++
PY ?= python
NCCL_INC ?= $(shell $(PY) -c "import nvidia.nccl,os;print(os.path.join(list(nvidia.nccl.__path__)[0],'include'))" 2>/dev/null || echo /usr/include)
OUT := scc26_nccl_shim_b200/lib
BUILD := _build
ARCH := -gencode arch=compute_100a,code=sm_100a

CORE_SRC := $(wildcard src/core/*.cc)
EXEC_SRC := $(wildcard src/exec/*.cc)
ABI_SRC := $(wildcard src/abi/*.cc)
CU_SRC := $(wildcard src/kernels/*.cu) $(wildcard src/exec/*.cu)
HDRS := $(wildcard src/*/*.h) $(wildcard src/*/*.cuh)

BUILD_ID := $(shell cat $(CORE_SRC) $(EXEC_SRC) $(ABI_SRC) $(CU_SRC) $(HDRS) | sha256sum | cut -c1-16)

CXXFLAGS := -O2 -std=c++17 -fPIC -Wall -Wextra -Wno-unused-parameter -Isrc -pthread
NVFLAGS := $(ARCH) -lineinfo -O3 -std=c++17 --fmad=false -Isrc -I$(NCCL_INC) -Xcompiler -fPIC

CORE_OBJ := $(patsubst src/%.cc,$(BUILD)/core_only/%.o,$(CORE_SRC))
LIB_CXX_OBJ := $(patsubst src/%.cc,$(BUILD)/lib/%.o,$(CORE_SRC) $(EXEC_SRC) $(ABI_SRC))
LIB_CU_OBJ := $(patsubst src/%.cu,$(BUILD)/lib/%.cu.o,$(CU_SRC))

all: $(OUT)/libnccl_b200.so $(OUT)/libnb_core.so

core: $(OUT)/libnb_core.so

$(BUILD)/core_only/%.o: src/%.cc $(HDRS)
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -c $< -o $@

$(BUILD)/lib/%.o: src/%.cc $(HDRS)
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -I$(CUDA)/include -I$(NCCL_INC) -DNB_BUILD_ID=\"$(BUILD_ID)\" -c $< -o $@

$(BUILD)/lib/%.cu.o: src/%.cu $(HDRS)
	@mkdir -p $(dir $@)
	$(NVCC) $(NVFLAGS) -c $< -o $@

$(OUT)/libnb_core.so: $(CORE_OBJ)
	@mkdir -p $(OUT)
	$(CXX) -shared -pthread -o $@ $^

# No DT_NEEDED on libnccl: the real library is found at run time
# (dlsym RTLD_NEXT, then the already-loaded libnccl.so.2).
$(OUT)/libnccl_b200.so: $(LIB_CXX_OBJ) $(LIB_CU_OBJ)
	@mkdir -p $(OUT)
	$(NVCC) $(ARCH) -shared --cudart shared -Xcompiler -pthread -o $@ $^ -ldl

# The core and a randomized self-test under AddressSanitizer + UBSan (CPU);
# SAN_CXX is a compiler whose runtime ships libasan/libubsan.
SAN_CXX ?= $(shell command -v /usr/bin/g++ || echo $(CXX))
SAN := -O1 -g -std=c++17 -Isrc -pthread -fsanitize=address,undefined -fno-sanitize-recover=all \
       -fno-omit-frame-pointer
sanitize: $(BUILD)/core_selftest_san

$(BUILD)/core_selftest_san: $(CORE_SRC) src/selftest/core_selftest.cc $(HDRS)
	@mkdir -p $(BUILD)
	$(SAN_CXX) $(SAN) -o $@ $(CORE_SRC) src/selftest/core_selftest.cc

clean:
	rm -rf $(BUILD)/core_only $(BUILD)/lib $(BUILD)/core_selftest_san $(OUT)/libnccl_b200.so \
	       $(OUT)/libnb_core.so

.PHONY: all core sanitize clean
