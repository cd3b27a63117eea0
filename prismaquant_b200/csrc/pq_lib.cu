// Single translation unit of libprismaquant_b200.so: the kernels share the
// device error word and the E8M0 tables without relocatable device code.
#include "pq_sweep.cu"
#include "pq_sweep_fast.cu"
#include "pq_pack.cu"
#include "pq_fisher.cu"
#include "pq_codebook.cu"
#include "pq_outerr.cu"
#include "pq_capi.cu"
#include "pq_noalloc.cu"
