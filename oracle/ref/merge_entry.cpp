// C entry point over the reference's diskann::merge_shards_gpu (DANCE
// src/gpu_merge.cu:351-871, declared in include/gpu_merge.h:13), so that
// tests/golden/make_golden_merge.py can call the unmodified reference merge
// through ctypes.  Checker only: nothing in the product links it.
#include <cstdint>

#include "gpu_merge.h"

extern "C" int ref_merge_shards_gpu(const char *vamana_prefix, const char *vamana_suffix, const char *idmaps_prefix,
                                    const char *idmaps_suffix, uint64_t nshards, uint32_t max_degree,
                                    const char *output_vamana, const char *medoids_file)
{
    return diskann::merge_shards_gpu(vamana_prefix, vamana_suffix, idmaps_prefix, idmaps_suffix, nshards, max_degree,
                                     output_vamana, medoids_file);
}
