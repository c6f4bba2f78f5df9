# Builds oracle/_ref/libref_struct.so from the reference's own structural
# sources (read in place, never copied) plus oracle/ref_wrap.cpp.
# TEST INFRASTRUCTURE ONLY. Needs the reference tree at REF (default
# /root/reference); the GPU machine uses the prebuilt library or skips.
REF ?= /root/reference
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
OUT := $(HERE)_ref
SRCS := $(REF)/src/backend/BinaryContraction.cpp $(REF)/src/backend/BinaryPrimitives.cpp \
        $(REF)/src/frontend/EinsumExpression.cpp $(REF)/src/frontend/EinsumExpressionAscii.cpp \
        $(REF)/src/frontend/EinsumTreeAscii.cpp $(HERE)ref_wrap.cpp
CXXFLAGS := -O1 -std=c++17 -fPIC -ffunction-sections -fdata-sections -fopenmp -w -I$(REF)/src

all: $(OUT)/libref_struct.so

$(OUT)/libref_struct.so: $(SRCS) $(HERE)ref.map
	mkdir -p $(OUT)
	g++ $(CXXFLAGS) -shared -Wl,--gc-sections -Wl,--version-script=$(HERE)ref.map -o $@ $(SRCS)

clean:
	rm -f $(OUT)/libref_struct.so

.PHONY: all clean
