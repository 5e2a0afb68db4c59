# Build: libq35cuda.so + engine (product) and libq35oracle.so (test oracle).
# sm_100a only. `make -j` from the repository root.
PKG      := enginesmith-qwen35-08b-long-decode-m5max-round005_b200
CSRC     := $(PKG)/csrc
LIBDIR   := $(PKG)/lib
BUILD    := _build
NVCC     ?= nvcc
CXX      ?= g++
ARCH     := -gencode arch=compute_100a,code=sm_100a
NVFLAGS  := -std=c++17 -O3 -lineinfo $(ARCH) -Xcompiler -fPIC -Iinclude -I$(CSRC)
CXXFLAGS := -std=c++17 -O2 -fPIC -Wall -Iinclude -I$(CSRC)

LIB      := $(LIBDIR)/libq35cuda.so
ENGINE   := $(LIBDIR)/engine
ORACLE   := oracle/libq35oracle.so

all: $(LIB) $(ENGINE) $(ORACLE)

$(BUILD)/%.o: $(CSRC)/%.cu $(wildcard $(CSRC)/*.cuh) $(wildcard $(CSRC)/*.h) include/q35.h
	@mkdir -p $(BUILD)
	$(NVCC) $(NVFLAGS) -c $< -o $@

$(BUILD)/q35_synth.o: $(CSRC)/q35_synth.cpp include/q35.h
	@mkdir -p $(BUILD)
	$(CXX) $(CXXFLAGS) -O3 -c $< -o $@

$(LIB): $(BUILD)/q35_kernels.o $(BUILD)/q35_prefill.o $(BUILD)/q35_gemm.o $(BUILD)/q35_tokens.o $(BUILD)/q35_prompt.o $(BUILD)/q35_runtime.o $(BUILD)/q35_noalloc.o $(BUILD)/q35_synth.o
	@mkdir -p $(LIBDIR)
	$(NVCC) $(ARCH) -shared -o $@ $^ -lcudart -lpthread

$(ENGINE): $(CSRC)/engine.cpp $(CSRC)/q35_json.h include/q35.h $(LIB)
	$(CXX) $(CXXFLAGS) -o $@ $< -L$(LIBDIR) -lq35cuda -Wl,-rpath,'$$ORIGIN' -pthread

# The oracle also carries the seeded synthetic-model writer (plain C++), so the
# CPU reference arm can write the model without loading the CUDA library.
$(ORACLE): oracle/q35_oracle.cpp oracle/q35_oracle.h $(CSRC)/q35_synth.cpp include/q35.h
	$(CXX) -std=c++17 -O2 -fPIC -shared -ffp-contract=off -pthread -Wall -Iinclude -o $@ oracle/q35_oracle.cpp $(CSRC)/q35_synth.cpp

clean:
	rm -rf $(BUILD) $(LIB) $(ENGINE) $(ORACLE)

.PHONY: all clean
