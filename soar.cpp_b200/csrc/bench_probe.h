/*
 * bench_probe.h -- measurement entry points of libsoar_probe.so, loaded only
 * by the bench. Not part of the optimizer library's C-ABI.
 */
#ifndef SOAR_BENCH_PROBE_H
#define SOAR_BENCH_PROBE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SOAR_PROBE_API __attribute__((visibility("default")))

/* The raw NVLink rate of the fused data-parallel step's two peer-memory access
   patterns, with no arithmetic, on symmetric buffers of at least
   world * bytes_per_peer bytes (bases[q]: rank q's, as seen from this process;
   16-byte aligned). Every rank calls it at once.
   mode 0 (pull, k_rs_sumsq's reads): bulk-loads bytes [rank * bytes_per_peer,
   (rank + 1) * bytes_per_peer) of every peer's buffer into a shared-memory
   ring of `stages` stages of tile_bytes per peer (stages * tile_bytes *
   (world - 1) <= 200 KB). mode 1 (push, k_apply's all-gather writes):
   bulk-stores zero tiles into that range of every peer's buffer (overwrites
   it). tile_bytes: a multiple of 16 dividing bytes_per_peer. `grid` CTAs.
   A wait that runs out (1 s) sets *d_err. Returns 0, or -1 with
   soar_probe_last_error() set. */
SOAR_PROBE_API int soar_nvlink_probe(void* const* bases, int world, int rank,
                                     uint64_t bytes_per_peer, int mode, uint32_t tile_bytes,
                                     int stages, int grid, int* d_err, void* stream);

/* Message of the calling thread's last failed probe call. */
SOAR_PROBE_API const char* soar_probe_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* SOAR_BENCH_PROBE_H */
