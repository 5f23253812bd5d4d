/* g4synth.h — seeded synthetic model images in the gemma4.c .bin layout. */
#ifndef G4SYNTH_H
#define G4SYNTH_H

#include <stdint.h>

#include "../csrc/g4_format.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Per-(row, 64-group) scale jitter in [0.5, 1.5) x base instead of one scale per row. */
#define G4SYN_GROUP_SCALES 1u
/* Norm weights and layer scalars uniform in [0.5, 1.5) instead of 1.0. */
#define G4SYN_RANDOM_NORMS 2u

/* Fills `records` (G4_NUM_RECORDS entries, offsets relative to the file start)
 * and returns the image size in bytes (5,008,891,264 for E2B). */
uint64_t g4synth_layout(g4_record *records);
uint64_t g4synth_image_bytes(void);
/* Writes a complete image into `image` (at least g4synth_image_bytes() bytes).
 * Returns 0 or a negative error. */
int g4synth_fill(uint8_t *image, uint64_t bytes, uint64_t seed, unsigned flags);
int g4synth_write_file(const char *path, uint64_t seed, unsigned flags);
uint16_t g4synth_f32_to_f16(float f);

#ifdef __cplusplus
}
#endif
#endif
