/* Compatibility name: adapters written against the reference include
 * "b3_batch.cuh" (B3Batch, b3_batch_step_gpu, b3_batch_restore_gpu); like the
 * reference's, it includes puffysics.cuh, which resolves to this library's
 * public header (plus, under nvcc, the device b3_step). */
#pragma once
#include "puffysics.cuh"
