// kvquant_b200: the whole library as one translation unit (no relocatable
// device code needed; the device status word has a single definition).
#include "kvq_common.cuh"
#include "kvq_runtime.cuh"
#include "kvq_ref_ops.cuh"
#include "kvq_quantize.cuh"
#include "kvq_append.cuh"
#include "kvq_decode.cuh"
#include "kvq_noalloc.cuh"
#include "kvq_codebook.cuh"
