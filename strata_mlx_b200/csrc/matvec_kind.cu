// The decode matvec variants of one block type; the build compiles this file once per type with -DMV_KIND=k.
#include "matvec_impl.cuh"

#ifndef MV_KIND
#error "compile with -DMV_KIND=<block type>"
#endif

template int sc::mv_dispatch<MV_KIND>(sc::MvArgs, int, int, int, int, cudaStream_t);
