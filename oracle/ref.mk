# ref.mk — compiles the reference's CPU path (songqiuyu/llm_core) IN PLACE from
# its own sources with g++, plus oracle/ref_harness.cpp, into
# oracle/_ref/libaxref.so.  Test infrastructure only.
#
#   make -f oracle/ref.mk REF=/path/to/reference      (from the repo root)
#
# Nothing is written outside oracle/_ref/.  The reference's CMake build is not
# used: the only file CMake would generate, include/axonforge/version.hpp, is
# written here as a four-macro stand-in (its template is
# include/axonforge/version.hpp.in).
REF      ?= ../reference
OUT      := oracle/_ref
OBJ      := $(OUT)/obj
CXX      ?= g++
CXXFLAGS := -std=c++20 -O3 -fPIC -DNDEBUG -pthread \
            -I$(REF)/include -I$(OUT)/include -I$(REF)/src -I$(REF)
AVX2     := -mavx2 -mfma -mf16c
VNNI     := -mavx2 -mfma -mf16c -mavxvnni
AVX512   := -mavx512f -mavx512vnni -mavx512bw

PLAIN_SRCS := src/engine.cpp src/core/graph.cpp src/core/tensor.cpp src/core/fuse_pass.cpp \
              src/core/liveness.cpp src/core/shape_infer.cpp src/backend/backend_registry.cpp \
              src/backend/cpu_x86/x86_backend.cpp src/backend/cpu_x86/cpu_arena.cpp \
              src/backend/cpu_x86/cpuid.cpp src/loader/gguf_loader.cpp \
              src/models/gpt2_model.cpp src/models/qwen2_model.cpp \
              src/models/hunyuan_dense_model.cpp src/tokenizer/bpe_tokenizer.cpp
AVX2_SRCS  := $(addprefix src/backend/cpu_x86/kernels/, gemm_avx2.cpp gemv_lut_avx2.cpp \
              gemv_f16_avx2.cpp gemv_q4k_avx2.cpp gemv_q6k_avx2.cpp quant_q8_avx2.cpp \
              gemv_q4k_q8_avx2.cpp gemv_q4k_r8_avx2.cpp gemv_q6k_q8_avx2.cpp \
              elementwise_avx2.cpp norm_avx2.cpp)
VNNI_SRCS  := $(addprefix src/backend/cpu_x86/kernels/, gemv_q4k_q8_avxvnni.cpp gemv_q4k_r8_avxvnni.cpp)
A512_SRCS  := $(addprefix src/backend/cpu_x86/kernels/, gemv_lut_avx512.cpp gemm_int8_vnni.cpp)

obj = $(patsubst %.cpp,$(OBJ)/%.o,$(subst /,_,$(1)))
PLAIN_OBJS := $(foreach s,$(PLAIN_SRCS),$(call obj,$(s)))
AVX2_OBJS  := $(foreach s,$(AVX2_SRCS),$(call obj,$(s)))
VNNI_OBJS  := $(foreach s,$(VNNI_SRCS),$(call obj,$(s)))
A512_OBJS  := $(foreach s,$(A512_SRCS),$(call obj,$(s)))
HARNESS    := $(OBJ)/ref_harness.o

all: $(OUT)/libaxref.so $(OUT)/libaxref_b200.so

$(OUT)/include/axonforge/version.hpp:
	@mkdir -p $(dir $@)
	@printf '#pragma once\n#define AXONFORGE_VERSION_MAJOR 0\n#define AXONFORGE_VERSION_MINOR 1\n#define AXONFORGE_VERSION_PATCH 0\n#define AXONFORGE_VERSION_STRING "0.1.0"\n' > $@

define compile_rule
$(call obj,$(1)): $(REF)/$(1) $(OUT)/include/axonforge/version.hpp
	@mkdir -p $(OBJ)
	$(CXX) $(CXXFLAGS) $(2) -c $$< -o $$@
endef
$(foreach s,$(PLAIN_SRCS),$(eval $(call compile_rule,$(s),)))
$(foreach s,$(AVX2_SRCS),$(eval $(call compile_rule,$(s),$(AVX2))))
$(foreach s,$(VNNI_SRCS),$(eval $(call compile_rule,$(s),$(VNNI))))
$(foreach s,$(A512_SRCS),$(eval $(call compile_rule,$(s),$(AVX512))))

# The harness #includes src/models/llama_model.cpp; it is compiled with the
# same flags the reference gives that file (no ISA flags: the model file uses
# AVX2 intrinsics through target attributes / the kernels it calls).
$(HARNESS): oracle/ref_harness.cpp $(REF)/src/models/llama_model.cpp $(OUT)/include/axonforge/version.hpp
	@mkdir -p $(OBJ)
	$(CXX) $(CXXFLAGS) $(AVX2) -c $< -o $@

$(OUT)/libaxref.so: $(PLAIN_OBJS) $(AVX2_OBJS) $(VNNI_OBJS) $(A512_OBJS) $(HARNESS)
	$(CXX) -shared -pthread -o $@ $^

.PHONY: all

# ---- the reference engine with the B200 path bound in (test infrastructure)
# llama_model.cpp compiled with AXONFORGE_HAS_CUDA (its llama_generate then
# dispatches backend "cuda" to llama_cuda_generate), the reference-side
# binding under integration/ (the "cuda" IBackend and llama_cuda_generate, in
# place of src/backend/cuda/* and src/models/llama_cuda_model.cpp) and
# oracle/integ_harness.cpp, linked with llm_core_b200/libaf_b200.so.
CUDA     ?= /usr/local/cuda
B200_LIB := llm_core_b200/libaf_b200.so
INTEG_FLAGS := -Iinclude -I$(CUDA)/include
INTEG_OBJS := $(OBJ)/integ_llama_model.o $(OBJ)/integ_af_cuda_backend.o $(OBJ)/integ_af_llama_cuda.o \
              $(OBJ)/integ_harness.o

$(OBJ)/integ_llama_model.o: $(REF)/src/models/llama_model.cpp $(OUT)/include/axonforge/version.hpp
	@mkdir -p $(OBJ)
	$(CXX) $(CXXFLAGS) $(AVX2) -DAXONFORGE_HAS_CUDA $(INTEG_FLAGS) -c $< -o $@

$(OBJ)/integ_%.o: integration/%.cpp include/af_b200.h $(OUT)/include/axonforge/version.hpp
	@mkdir -p $(OBJ)
	$(CXX) $(CXXFLAGS) $(INTEG_FLAGS) -c $< -o $@

$(OBJ)/integ_harness.o: oracle/integ_harness.cpp $(OUT)/include/axonforge/version.hpp
	@mkdir -p $(OBJ)
	$(CXX) $(CXXFLAGS) $(INTEG_FLAGS) -c $< -o $@

$(OUT)/libaxref_b200.so: $(PLAIN_OBJS) $(AVX2_OBJS) $(VNNI_OBJS) $(A512_OBJS) $(INTEG_OBJS) $(B200_LIB)
	$(CXX) -shared -pthread -o $@ $(filter %.o,$^) -Lllm_core_b200 -l:libaf_b200.so -L$(CUDA)/lib64 -lcudart \
	    -Wl,-rpath,'$$ORIGIN/../../llm_core_b200'
