// Persistent decode-step kernel instantiation: rows up to 4096 elements
// (16 input chunks per lane), sliding layers head_dim 256 with 2 query heads per KV
// head, full layers head_dim 512 with 8 (the real checkpoint's global layers at world 1,
// whose 8192-element o_proj rows run as two sub-rows).
#include "g4_step.cuh"

G4_STEP_VARIANT(16, 256, 2, 512, 8)
