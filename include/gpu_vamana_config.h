/*
 * gpu_vamana_config.h -- build knobs of the standard builder.
 *
 * The reference fixes these at compile time (include/gpu_vamana_config.h and
 * the CMake DANCE_PROFILE presets in the DiskANN integration patch, lines
 * 2398-2450).  The macro names and release values are kept so that a build
 * configured with -D<NAME>=<value> behaves the same; libdance_b200.so reads
 * them as the DEFAULTS of a runtime parameter block (DanceVamanaParams in
 * dance_b200.h), so tests can also vary them per call.
 */
#ifndef DANCE_B200_GPU_VAMANA_CONFIG_H
#define DANCE_B200_GPU_VAMANA_CONFIG_H

#ifndef DANCE_PROFILE_NAME
#define DANCE_PROFILE_NAME "QUALITY"
#endif

/* Synchronous refinement rounds (reference config line "VAMANA_ITERS 4"). */
#ifndef VAMANA_ITERS
#define VAMANA_ITERS 4
#endif

/* alpha of the last round; earlier rounds use 1.0
 * (reference src/gpu_vamana_vnew2.cu:201-213). */
#ifndef VAMANA_ALPHA
#define VAMANA_ALPHA 1.2f
#endif

/* Float input is stored and searched as fp16 when 1 (FAST_SMALL profile). */
#ifndef ENABLE_FLOAT16_BUILD
#define ENABLE_FLOAT16_BUILD 0
#endif

/* Hash seeds added to every vertex search (config INIT_RANDOM_SEEDS). */
#ifndef INIT_RANDOM_SEEDS
#define INIT_RANDOM_SEEDS 8
#endif

/* Last round refills each row to min(FINAL_MIN_DEGREE, R) with the nearest
 * unselected candidates (config ENABLE_FINAL_DEGREE_FILL / FINAL_MIN_DEGREE). */
#ifndef ENABLE_FINAL_DEGREE_FILL
#define ENABLE_FINAL_DEGREE_FILL 1
#endif
#ifndef FINAL_MIN_DEGREE
#define FINAL_MIN_DEGREE 64
#endif

/* Approximate medoid: candidates x samples (config MEDOID_NUM_*). */
#ifndef MEDOID_NUM_CANDIDATES
#define MEDOID_NUM_CANDIDATES 1024
#endif
#ifndef MEDOID_NUM_SAMPLES
#define MEDOID_NUM_SAMPLES 4096
#endif

/* First COARSE_WARMUP_ITERS rounds cap the expansion steps at
 * WARMUP_EXPAND_STEPS (config ENABLE_COARSE_TO_FINE_STEPS). */
#ifndef ENABLE_COARSE_TO_FINE_STEPS
#define ENABLE_COARSE_TO_FINE_STEPS 1
#endif
#ifndef COARSE_WARMUP_ITERS
#define COARSE_WARMUP_ITERS 2
#endif
#ifndef WARMUP_EXPAND_STEPS
#define WARMUP_EXPAND_STEPS 64
#endif

/* Reverse merge heavy-row cap: rows with more than REVERSE_HEAVY_THRESHOLD
 * reverse sources only look at REVERSE_HEAVY_SAMPLE evenly spaced ones
 * (PRO6000_100M and FILTERED_PAPER profiles). */
#ifndef ENABLE_REVERSE_HEAVY_CAP
#define ENABLE_REVERSE_HEAVY_CAP 0
#endif
#ifndef REVERSE_HEAVY_THRESHOLD
#define REVERSE_HEAVY_THRESHOLD 256
#endif
#ifndef REVERSE_HEAVY_SAMPLE
#define REVERSE_HEAVY_SAMPLE 256
#endif

#endif /* DANCE_B200_GPU_VAMANA_CONFIG_H */
