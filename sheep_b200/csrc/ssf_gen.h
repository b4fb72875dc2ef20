// Seeded synthetic SSF model writer (see ssf_gen.c). The spec struct and the
// entry point are declared in sheep_b200.h.
#pragma once

#include <stdint.h>

#include "sheep_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

uint16_t ssfgen_f32_to_f16(float f);
float    ssfgen_f16_to_f32(uint16_t h);

#ifdef __cplusplus
}
#endif
