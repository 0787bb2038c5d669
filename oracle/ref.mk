# Builds the reference's own CUDA launchers (acediaR src/kernels/tensor_ops.cu
# and tensor_kernels.cu, compiled where they lie, unmodified) into
# oracle/_ref/libacediar_ref.so.  Test infrastructure only: the GPU tests use
# it to pin the CPU oracle against the reference's own results on small
# inputs.  Needs the reference sources (present only on the build machine);
# the built library travels with the repository snapshot.
# REF: the reference checkout's src/ directory (make REF=...); by default
# $(ACEDIAR_REF)/src, with ACEDIAR_REF defaulting to the build machine's copy
ACEDIAR_REF ?= /root/reference
REF ?= $(ACEDIAR_REF)/src
NVCC ?= nvcc
OUT := _ref/libacediar_ref.so

all: $(OUT)

$(OUT): $(REF)/kernels/tensor_ops.cu $(REF)/kernels/tensor_kernels.cu
	mkdir -p _ref
	$(NVCC) -O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC -shared \
	  -I$(REF)/kernels -I$(REF) $(REF)/kernels/tensor_ops.cu $(REF)/kernels/tensor_kernels.cu \
	  -o $@ -lcublas -Xlinker -Bsymbolic

clean:
	rm -rf _ref

.PHONY: all clean
