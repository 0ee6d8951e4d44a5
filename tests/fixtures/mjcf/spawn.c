/* Loads an MJCF file with the reference's loader (mjcf.h), spawns it into a
 * B3World with a ground and applies a keyframe, and writes the world's bytes:
 *     spawn <model.xml> <key or -> <out.bin>
 * The MJCF scene-ingestion tests compile this file twice, against the
 * reference's physics headers and against this library's include/ (the
 * loader itself only uses the public world-building API). */
#include <stdio.h>

#include "mjcf.h"

static MjcfModel model;
static B3World world;

int main(int argc, char** argv) {
    if (argc < 4) return 2;
    if (!mjcf_load(&model, argv[1], 1)) {
        fprintf(stderr, "%s\n", model.error);
        return 3;
    }
    b3_world_init(&world);
    world.gravity = b3_v(0.0f, -9.81f, 0.0f);
    MjcfSpawn s;
    if (!mjcf_spawn(&model, &world, &s, 1)) return 4;
    if (argv[2][0] != '-' && !mjcf_apply_key(&world, &model, &s, argv[2])) return 5;
    FILE* f = fopen(argv[3], "wb");
    if (!f) return 6;
    size_t n = fwrite(&world, sizeof(world), 1, f);
    fclose(f);
    mjcf_free(&model);
    printf("%d %d %d %d\n", world.body_count, world.shape_count, world.joint_count, b3_world_error(&world));
    return n == 1 ? 0 : 7;
}
