/* Compatibility name: adapters written against the reference include
 * "puffysics.cuh"; it resolves to this library's public header. */
#pragma once
#include "puffysics_b200.h"
