/* b3_test_forces.h -- a per-substep force hook for the parity tests of the
 * reference's B3_USER_FORCES mode (src/puffysics/01_config.inl:186-198).
 *
 * Pulls every dynamic body toward (0, 2, 0) by its current center (center +
 * delta_pos, as the reference's hook contract asks) and adds a constant spin
 * torque about y.  Given to the compiler with -include, before the physics
 * headers, in the same text for the reference's build, the CPU restatement
 * and this library's per-thread step.
 */
#pragma once
#define B3_USER_FORCES(w, h)                                                                       \
    do {                                                                                           \
        (void)(h);                                                                                 \
        for (int b3t_i = 0; b3t_i < (w)->body_count; b3t_i++) {                                    \
            B3Body* b3t_b = &(w)->bodies[b3t_i];                                                   \
            if (b3t_b->type != B3_DYNAMIC) continue;                                               \
            B3Vec3 b3t_p = b3_add(b3t_b->center, b3t_b->delta_pos);                                \
            b3t_b->force = b3_add(b3t_b->force,                                                    \
                b3_v(-3.0f * b3t_p.x, 3.0f * (2.0f - b3t_p.y), -3.0f * b3t_p.z));                  \
            b3t_b->torque = b3_add(b3t_b->torque, b3_v(0.0f, 0.5f, 0.0f));                         \
        }                                                                                          \
    } while (0)
