/* Compatibility name: adapters written against the reference include
 * "b3_batch.cuh" (B3Batch, b3_batch_step_gpu, b3_batch_restore_gpu); it
 * resolves to this library's public header. */
#pragma once
#include "puffysics_b200.h"
