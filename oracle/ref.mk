# Builds, from the reference's own sources (read in place, never copied),
#   oracle/_ref/libref_struct.so  structural host functions (+ ref_wrap.cpp)
#   oracle/_ref/libref_scalar.so  the scalar contraction / permute backends
#                                 (+ ref_scalar.cpp, stub/libxsmm.h)
# TEST INFRASTRUCTURE ONLY. REF must name the reference checkout (the
# directory holding src/); there is no default. The GPU machine uses the
# prebuilt libraries or skips the tests that need them.
ifndef REF
$(error REF is not set: pass REF=<reference checkout> (the directory holding src/))
endif
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
OUT := $(HERE)_ref
S := $(REF)/src
STRUCT_SRCS := $(S)/backend/BinaryContraction.cpp $(S)/backend/BinaryPrimitives.cpp \
        $(S)/frontend/EinsumExpression.cpp $(S)/frontend/EinsumExpressionAscii.cpp \
        $(S)/frontend/EinsumTreeAscii.cpp $(HERE)ref_wrap.cpp
SCALAR_SRCS := $(S)/backend/BinaryContraction.cpp $(S)/backend/BinaryContractionScalar.cpp \
        $(S)/backend/MemoryManager.cpp $(S)/backend/Unary.cpp $(S)/backend/UnaryScalar.cpp \
        $(S)/basic/binary/ContractionBackend.cpp $(S)/basic/binary/ContractionBackendScalar.cpp \
        $(S)/basic/binary/ContractionOptimizer.cpp $(S)/basic/binary/ContractionMemoryManager.cpp \
        $(S)/basic/binary/IterationSpace.cpp $(S)/basic/unary/UnaryBackend.cpp \
        $(S)/basic/unary/UnaryBackendScalar.cpp $(S)/basic/unary/UnaryOptimizer.cpp \
        $(HERE)ref_scalar.cpp
CXXFLAGS := -O1 -std=c++17 -fPIC -ffunction-sections -fdata-sections -fopenmp -w -I$(S)
# the reference's release flags (SConstruct: -O2, OpenMP)
SCALAR_FLAGS := -O2 -std=c++17 -fPIC -fopenmp -w -I$(S) -I$(HERE)stub

all: $(OUT)/libref_struct.so $(OUT)/libref_scalar.so

$(OUT)/libref_struct.so: $(STRUCT_SRCS) $(HERE)ref.map
	mkdir -p $(OUT)
	g++ $(CXXFLAGS) -shared -Wl,--gc-sections -Wl,--version-script=$(HERE)ref.map -o $@ $(STRUCT_SRCS)

$(OUT)/libref_scalar.so: $(SCALAR_SRCS) $(HERE)stub/libxsmm.h $(HERE)ref.map
	mkdir -p $(OUT)
	g++ $(SCALAR_FLAGS) -shared -Wl,--version-script=$(HERE)ref.map -o $@ $(SCALAR_SRCS)

clean:
	rm -f $(OUT)/libref_struct.so $(OUT)/libref_scalar.so

.PHONY: all clean
