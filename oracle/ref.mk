# ref.mk -- TEST INFRASTRUCTURE: builds reference-side checkers into oracle/_ref/ (git-ignored; the built binaries
# travel to the GPU box, the reference tree does not).  Run from anywhere:  make -f oracle/ref.mk [REF=...]
#
#   _ref/emu_dump      the reference's Hopper host emulator (hopper/emu/emu.cpp, compiled where it lies) driven by
#                      oracle/ref_emu_dump.cpp: dumps one reference kernel's inputs, fp64 reference and C (CPU only)
#   _ref/verif_bw      the reference's own GPU check, hopper/verif.cu compiled where it lies, linked with this
#                      repository's candidate (gemm-ladder_b200/blackwell/candidate.cu, the whole rung in one
#                      translation unit): the reference's 26 edge shapes, its fp64 CPU reference and its 8
#                      bit-for-bit repeats of every variant, run on the B200
#   _ref/judge_bw      the reference's judge, judge/judge.cu compiled where it lies (force-including
#                      oracle/judge_compat.h so that CUDA 12.9 builds it) and linked with this repository's candidate,
#                      with its inputs: _ref/shapes_b200.txt (the judge's 17 B200 shapes, written from tests/shapes.py
#                      in the judge's "M N K label" format) and _ref/judge_reference_b200.txt (the card's cached
#                      cuBLASLt configurations, judge/reference/b200.txt, data read by --reference)
#   _ref/probe_bw      the reference's probe, probe/probe.cu compiled where it lies (force-including
#                      oracle/judge_compat.h: it takes the same four CUDA 13 graph calls, probe/probe.cu:162-177) and
#                      linked with this repository's candidate: interleaved timing of the arms v<i>, twin and x:<hex>
#
# Nothing here is built from a copy of the reference's sources, and nothing runs the reference's own build system.
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
ROOT := $(abspath $(HERE)..)
# the reference project's tree: REF=<path>, else a checkout named "reference" beside this repository
REF ?= $(abspath $(ROOT)/../reference)
OUT := $(HERE)_ref
CXX ?= g++
NVCC ?= nvcc
PKG := $(ROOT)/gemm-ladder_b200

all: $(OUT)/emu_dump $(OUT)/verif_bw judge_bw $(OUT)/probe_bw
emu_dump: $(OUT)/emu_dump
verif_bw: $(OUT)/verif_bw
probe_bw: $(OUT)/probe_bw
judge_bw: $(OUT)/judge_bw $(OUT)/shapes_b200.txt $(OUT)/judge_reference_b200.txt

$(OUT):
	mkdir -p $(OUT)

$(OUT)/emu_dump: $(HERE)ref_emu_dump.cpp | $(OUT)
	$(CXX) -std=c++17 -O2 -march=x86-64-v3 -w -I$(REF)/hopper/emu -I$(REF)/hopper -I$(REF)/hopper/emu/shim \
	    $(HERE)ref_emu_dump.cpp -o $@

$(OUT)/verif_bw: $(REF)/hopper/verif.cu $(PKG)/blackwell/candidate.cu $(wildcard $(PKG)/csrc/*) | $(OUT)
	$(NVCC) -std=c++17 -O2 -gencode arch=compute_100a,code=sm_100a -I$(ROOT)/include \
	    $(REF)/hopper/verif.cu $(PKG)/blackwell/candidate.cu -o $@ -lcublasLt

$(OUT)/judge_bw: $(REF)/judge/judge.cu $(HERE)judge_compat.h $(PKG)/blackwell/candidate.cu $(wildcard $(PKG)/csrc/*) | $(OUT)
	$(NVCC) -std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a -I$(ROOT)/include -include $(HERE)judge_compat.h \
	    $(REF)/judge/judge.cu $(PKG)/blackwell/candidate.cu -o $@ -lcublasLt -lcublas

$(OUT)/probe_bw: $(REF)/probe/probe.cu $(HERE)judge_compat.h $(PKG)/blackwell/candidate.cu $(wildcard $(PKG)/csrc/*) | $(OUT)
	$(NVCC) -std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a -I$(ROOT)/include -include $(HERE)judge_compat.h \
	    $(REF)/probe/probe.cu $(PKG)/blackwell/candidate.cu -o $@ -lcublasLt -lcublas

$(OUT)/shapes_b200.txt: $(ROOT)/tests/shapes.py | $(OUT)
	cd $(ROOT)/tests && python3 -c "from shapes import JUDGE_B200; print('# M N K label'); \
	    [print(m, n, k, name) for name, m, n, k in JUDGE_B200]" > $@

$(OUT)/judge_reference_b200.txt: $(REF)/judge/reference/b200.txt | $(OUT)
	cp $< $@

.PHONY: all emu_dump verif_bw judge_bw probe_bw
