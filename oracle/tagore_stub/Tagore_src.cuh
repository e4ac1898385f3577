// TEST INFRASTRUCTURE ONLY -- stand-in for the external Tagore library header that
// UNG/codes/src/tagore_graph_builder.cu includes.  That library (GNN descent and its
// helpers) is not part of the reference tree, so this header only makes the file
// compile: constants for its shared arrays and buffer sizes, and no-op placeholders
// for the kernels and device functions of the GNN-descent route.  The checker
// (oracle/knn_ref_harness.cpp) calls only the route that groups up to the
// fast-exact threshold take -- build_fast_exact_cuda_batch and its
// batched_exact_knn_graph_kernel, both defined in the reference file itself -- so no
// placeholder here is ever executed.
#pragma once

#include <iostream>

#define FINAL_DEGREE_SIZE 128
#define RESERVENUM 64
#define SAMPLE 16
#define MAX_P 128
#define SELECT_CAND 16

typedef float (*funcFormat)(const float *, const float *, unsigned);

__device__ inline float distance_filter(const float *, const float *, unsigned) { return 0.0f; }

template <class... A>
__device__ void bitonic_sort_id_and_dis(A...)
{
}

#define UNGX_TAGORE_PLACEHOLDER_KERNEL(name)                                                                          \
   template <class... A>                                                                                         \
   __global__ void name(A...)                                                                                    \
   {                                                                                                             \
   }

UNGX_TAGORE_PLACEHOLDER_KERNEL(initialize_graph)
UNGX_TAGORE_PLACEHOLDER_KERNEL(cal_power)
UNGX_TAGORE_PLACEHOLDER_KERNEL(nn_descent_opt_sample)
UNGX_TAGORE_PLACEHOLDER_KERNEL(nn_descent_opt_reverse_sample)
UNGX_TAGORE_PLACEHOLDER_KERNEL(reset_reverse_new_old_num)
UNGX_TAGORE_PLACEHOLDER_KERNEL(nn_descent_opt_cal)
UNGX_TAGORE_PLACEHOLDER_KERNEL(nn_descent_opt_merge)
UNGX_TAGORE_PLACEHOLDER_KERNEL(reset_reverse_num)
UNGX_TAGORE_PLACEHOLDER_KERNEL(do_reverse_graph)
UNGX_TAGORE_PLACEHOLDER_KERNEL(reset_visit_reversenum)
UNGX_TAGORE_PLACEHOLDER_KERNEL(sample_kernel6)
UNGX_TAGORE_PLACEHOLDER_KERNEL(merge_reverse_plus)
UNGX_TAGORE_PLACEHOLDER_KERNEL(cal_ep_gpu)
UNGX_TAGORE_PLACEHOLDER_KERNEL(select_path)
UNGX_TAGORE_PLACEHOLDER_KERNEL(filter_reverse)

#undef UNGX_TAGORE_PLACEHOLDER_KERNEL
