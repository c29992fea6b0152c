// Persistent decode-step kernel instantiation: rows up to 3072 elements
// (12 input chunks per lane), sliding layers head_dim 256 with 2 query heads per KV
// head, full layers head_dim 512 with 1 (per rank).
#include "g4_step.cuh"

G4_STEP_VARIANT(12, 256, 2, 512, 1)
