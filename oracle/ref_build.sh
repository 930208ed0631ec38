#!/usr/bin/env bash
# Compiles the reference's own CPU integrator from its sources (read-only,
# under the reference tree) into oracle/_ref/hxref_run -- TEST INFRASTRUCTURE
# ONLY (the checker that pins oracle/hx_oracle.c).  No reference file is copied;
# only the HighFive type shim (oracle/ref_shim) and the harness
# (oracle/ref_harness.cpp) are ours.  Flags follow the reference's
# CMakeLists.txt:7-31 (C++20, -ffp-contract=off, -fno-fast-math).
set -euo pipefail
HERE=$(cd "$(dirname "$0")" && pwd)
# the reference checkout: HX_REFERENCE, else the one beside this repository
REF=${HX_REFERENCE:-$HERE/../../reference}/src
OUT=$HERE/_ref
OBJ=$OUT/obj
mkdir -p "$OBJ"
if [ ! -d "$REF" ]; then echo "reference sources not found: $REF" >&2; exit 1; fi

INC="-I$HERE/ref_shim -I/usr/local/cuda/include -I$REF -I$REF/io -I$REF/mech -I$REF/mech/build-in-mech -I$REF/mech/user-mech \
 -I$REF/mech/worm-mech -I$REF/mech/worm-lr-mech -I$REF/utils -I$REF/spike -I$REF/spike/postsyn_mech \
 -I$REF/spike/user_postsyn_mech -I$REF/third_party/CXXOPTS -I$REF/third_party/magic_enum -I$REF/third_party/Random123"
CXXFLAGS="-std=c++20 -O2 -fPIC -ffp-contract=off -fno-fast-math -fexcess-precision=standard -w"
NVFLAGS="-std=c++20 -O2 -Xcompiler -fPIC,-ffp-contract=off,-fno-fast-math,-w -diag-suppress=20040,177,550,186 -w \
 -gencode arch=compute_100a,code=sm_100a"

# the integrator, its loader and the mechanisms the synthetic configurations use
# (the library cells add the user-mech channel set and calcium dynamics)
SRCS=$(cd "$REF" && ls \
  simulate.cpp simulate.cu neuron.cpp permute.cpp permute_order.cpp vecplay.cu \
  io/*.cpp io/*.cu utils/*.cpp utils/*.cu mech/*.cpp mech/*.cu mech/build-in-mech/*.cpp mech/build-in-mech/*.cu \
  spike/*.cpp spike/*.cu spike/postsyn_mech/*.cpp spike/postsyn_mech/*.cu optimizer/*.cpp optimizer/*.cu \
  mech/user-mech/hh_templated.cu mech/user-mech/pas_templated.cu mech/user-mech/iclamp_templated.cu \
  mech/user-mech/HalfGap.cu mech/worm-lr-mech/gapjunction_lr.cu mech/worm-lr-mech/neuron_to_neuron_syn_lr.cu \
  mech/user-mech/CaDynamics_E2.cu mech/user-mech/CA_HVA.cu mech/user-mech/Ca_LVAst.cu mech/user-mech/Im.cu \
  mech/user-mech/K_Pst.cu mech/user-mech/K_Tst.cu mech/user-mech/NaTg.cu mech/user-mech/Nap_Et2.cu \
  mech/user-mech/SK_E2.cu mech/user-mech/SKv3_1.cu mech/user-mech/hd_la.cu mech/user-mech/km_la.cu \
  mech/user-mech/kca_la.cu mech/user-mech/it2_la.cu mech/user-mech/kdr_la.cu mech/user-mech/sca_la.cu \
  mech/user-mech/Ca.cu mech/worm-lr-mech/shl1_lr.cu mech/worm-lr-mech/kvs1_lr.cu mech/worm-lr-mech/irk_lr.cu \
  mech/worm-lr-mech/egl36_lr.cu mech/worm-lr-mech/shk1_lr.cu mech/worm-lr-mech/egl2_lr.cu \
  mech/worm-lr-mech/cca1_lr.cu mech/worm-lr-mech/egl19_lr.cu mech/worm-lr-mech/unc2_lr.cu \
  mech/worm-lr-mech/kcnl_lr.cu mech/worm-lr-mech/nca_lr.cu mech/worm-lr-mech/kqt3_lr.cu \
  mech/worm-lr-mech/cainternm_lr.cu mech/worm-mech/shl1.cu mech/worm-mech/kvs1.cu mech/worm-mech/irk.cu \
  mech/worm-mech/egl36.cu mech/worm-mech/shk1.cu mech/worm-mech/egl2.cu mech/worm-mech/cca1.cu \
  mech/worm-mech/egl19.cu mech/worm-mech/unc2.cu mech/worm-mech/gapjunction_noptr.cu \
  2>/dev/null)

compile() {
  src=$1
  obj=$OBJ/$(echo "$src" | tr '/' '_').o
  if [ -f "$obj" ] && [ "$obj" -nt "$REF/$src" ]; then return 0; fi
  case "$src" in
    *.cu) nvcc $NVFLAGS $INC -c "$REF/$src" -o "$obj" ;;
    *) g++ $CXXFLAGS $INC -c "$REF/$src" -o "$obj" ;;
  esac
}
export -f compile
export REF OBJ INC CXXFLAGS NVFLAGS
echo "$SRCS" | xargs -P "$(nproc)" -I{} bash -c 'compile {}'

g++ $CXXFLAGS $INC -c "$HERE/ref_harness.cpp" -o "$OBJ/_harness.o"
g++ $CXXFLAGS -I/usr/local/cuda/include -c "$HERE/ref_nodev.cpp" -o "$OBJ/_nodev.o"
# shared CUDA runtime, so that the host-only definitions in _nodev.o take precedence
nvcc -gencode arch=compute_100a,code=sm_100a -o "$OUT/hxref_run" "$OBJ"/*.o -cudart shared -lpthread \
  -Xlinker -rpath=/usr/local/cuda/lib64
# the same integrator against the real CUDA runtime: the reference's GPU path
nvcc -gencode arch=compute_100a,code=sm_100a -o "$OUT/hxref_run_gpu" $(ls "$OBJ"/*.o | grep -v '/_nodev.o$') \
  -cudart shared -lpthread -Xlinker -rpath=/usr/local/cuda/lib64
echo "built $OUT/hxref_run $OUT/hxref_run_gpu"
