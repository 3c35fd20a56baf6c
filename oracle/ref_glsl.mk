# Compiles the reference's hot-path GLSL shaders as C++ (test infrastructure).
#   make -C oracle -f ref_glsl.mk [REF=/path/to/reference]
# Reads shaders/*.comp from the reference tree where they lie, preprocesses
# them with ref_glsl.sed into _ref/*.inc and builds _ref/libref_glsl.so.
# Output goes only to oracle/_ref/ (git-ignored).  The reference tree is
# $STYX_REFERENCE_ROOT, else a "reference" folder beside this repository.
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
REF ?= $(or $(STYX_REFERENCE_ROOT),$(abspath $(HERE)../../reference))
OUT := $(HERE)_ref
CXX := $(firstword $(wildcard /usr/bin/g++) g++)
SHADERS := matvec_strided_f32 topk_softmax_f32 moe_reduce_f32 gather_slabs_f32 attn_decode_f32 add_flat_f32
INCS := $(addprefix $(OUT)/,$(addsuffix .inc,$(SHADERS)))

all: $(OUT)/libref_glsl.so

$(OUT)/%.inc: $(REF)/shaders/%.comp $(HERE)ref_glsl.sed
	@mkdir -p $(OUT)
	sed -E -f $(HERE)ref_glsl.sed $< > $@

$(OUT)/libref_glsl.so: $(HERE)ref_glsl.cpp $(HERE)ref_glsl_shim.h $(INCS)
	$(CXX) -O2 -fPIC -shared -fopenmp -ffp-contract=off -std=c++17 -Wno-attributes \
	    -I$(HERE) -I$(OUT) -o $@ $(HERE)ref_glsl.cpp

clean:
	rm -rf $(OUT)

.PHONY: all clean
