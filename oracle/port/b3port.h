/*
 * b3port.h -- CPU restatement of the Puffysics stepping path (parity oracle).
 * TEST INFRASTRUCTURE, NOT PRODUCT CODE: see b3port.c.
 * Include puffysics_b200.h (with the build's B3_MAX_* capacities) first.
 */
#ifndef B3PORT_H
#define B3PORT_H
void b3port_step(B3World* w, float dt, int substeps, int joint_iters, int relax_iters);
int b3port_batch_step(B3Batch batch, float dt, int substeps, const unsigned char* active,
    int joint_iters, int relax_iters);
int b3port_batch_restore(B3Batch batch, const B3World* initial, const unsigned char* reset);
int b3port_collide(const B3World* w, int shape_a, int shape_b, float* normal, float* pa, float* pb,
    float* sep, unsigned* feature);
#endif
