/*
 * gpu_merge.h -- GPU merge of overlapping shard graphs (drop-in for DANCE's
 * include/gpu_merge.h:13, called from DiskANN's merge_shards, integration
 * patch lines 3015-3035).
 *
 * Reads shard graphs <vamana_prefix>i<vamana_suffix> and id maps
 * <idmaps_prefix>i<idmaps_suffix> for i < nshards, writes the merged DiskANN
 * graph to output_vamana (each source keeps its first max_degree distinct
 * destinations in hash_edge32 rank order) and the medoids file.  Returns 0,
 * or the reference's negative code of the failing step: -2 id map, -3 graph
 * header / frozen points, -4 medoid out of range, -6 graph read, -7
 * neighbour out of range, -10 medoids file, -11 output file, -12 device,
 * -14..-17 device memory / copies / kernels, -19 degree overflow.
 * DISKANN_GPU_MERGE_DEVICES, DISKANN_GPU_MERGE_BUCKETS,
 * DISKANN_GPU_MERGE_BUCKET_EDGES and DISKANN_GPU_MERGE_HASH_SEED are honoured.
 */
#pragma once

#include <cstdint>
#include <string>

#ifndef DANCE_API
#define DANCE_API __attribute__((visibility("default")))
#endif

namespace diskann
{

DANCE_API int merge_shards_gpu(const std::string &vamana_prefix, const std::string &vamana_suffix,
                               const std::string &idmaps_prefix, const std::string &idmaps_suffix, uint64_t nshards,
                               uint32_t max_degree, const std::string &output_vamana,
                               const std::string &medoids_file);

}
