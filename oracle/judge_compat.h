/* judge_compat.h -- test infrastructure: lets the reference's judge (judge/judge.cu, which needs CUDA >= 13 for the
 * edge-data forms of four graph calls, judge/judge.cu:351-365) build unchanged with CUDA 12.x, force-included ahead of
 * it (nvcc -include oracle/judge_compat.h judge/judge.cu ...; recipe: oracle/ref.mk, target judge_bw).
 *
 * CUDA 12.3+ has the same four functions with the same parameters under versioned names; CUDA 13 gave them the plain
 * names.  The runtime header is included first, so that its own declarations keep their names, then the plain names
 * used by the judge are mapped onto the versioned ones.  Nothing else changes.
 */
#ifndef BW_JUDGE_COMPAT_H
#define BW_JUDGE_COMPAT_H
#include <cuda_runtime.h>
#if defined(CUDART_VERSION) && CUDART_VERSION < 13000
#undef cudaStreamGetCaptureInfo /* 12.x names its per-thread variant through a macro of this name */
#undef cudaGraphGetEdges
#undef cudaGraphRemoveDependencies
#undef cudaGraphAddDependencies
#define cudaStreamGetCaptureInfo cudaStreamGetCaptureInfo_v3
#define cudaGraphGetEdges cudaGraphGetEdges_v2
#define cudaGraphRemoveDependencies cudaGraphRemoveDependencies_v2
#define cudaGraphAddDependencies cudaGraphAddDependencies_v2
#endif
#endif
