/* frc_units.h - internal helpers of the unit-file loader (frc_units.c),
 * shared with frc.cu.  Not part of the public ABI. */
#ifndef FRC_UNITS_H
#define FRC_UNITS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Maps unit-BB.bin of `directory` read-only once unit-BB.sha256 is well
 * formed, the file has want_bytes (0: any size) and, with verify, its SHA-256
 * matches the recorded digest.  On success *data / *len hold the mapping
 * (release it with frc_unit_unmap); on failure a message goes to why. */
int frc_unit_map(const char *directory, unsigned block, uint64_t want_bytes, int verify, const void **data,
                 size_t *len, char *why, size_t why_len);
void frc_unit_unmap(const void *data, size_t len);

#ifdef __cplusplus
}
#endif

#endif
