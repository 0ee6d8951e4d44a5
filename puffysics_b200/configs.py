"""The benchmark configurations (BASELINE.json configs[0..4]) as data.

Each entry names the scene generator (puffysics_b200/scenes/b3_scenes.h),
capacities (B3_MAX_BODIES/SHAPES/CONTACTS/JOINTS), joint/relax iteration
counts, timestep, substeps and the world count of the configuration.
"""
from dataclasses import dataclass

SCENE_HOVER, SCENE_STACK, SCENE_CHAIN, SCENE_PILE, SCENE_BOUNCE, SCENE_CAPSULE = 1, 2, 3, 4, 5, 6
ACT_NONE, ACT_FORCE, ACT_TORQUE, ACT_LINEAR_IMPULSE, ACT_JOINT_TARGET = -1, 0, 1, 2, 3
STEP_INTERLEAVE_CONTACTS, STEP_SKIP_RESTITUTION = 1, 2


@dataclass(frozen=True)
class Config:
    name: str            # also the oracle library tag (libb3ref_<name>.so)
    scene: int
    caps: tuple          # (bodies, shapes, contacts, joints)
    joint_iters: int
    relax_iters: int
    dt: float
    substeps: int
    worlds: int
    steps: int = 0       # rollout length the configuration is quoted at (0 = open-ended)
    reset_fraction: float = 0.0
    description: str = ""
    flags: int = 0       # STEP_INTERLEAVE_CONTACTS | STEP_SKIP_RESTITUTION (the reference's mode macros)

    @property
    def signature(self):
        b, s, c, j = self.caps
        return b | (s << 16) | (c << 32) | (j << 48)

    @property
    def action(self):
        """(kind, first index, values per world) of the per-step action."""
        return {SCENE_HOVER: (ACT_FORCE, 1, 3),
                SCENE_STACK: (ACT_LINEAR_IMPULSE, 8, 3),
                SCENE_CHAIN: (ACT_JOINT_TARGET, 1, 9)}.get(self.scene, (ACT_NONE, 0, 0))


CONFIGS = {
    "hover": Config("hover", SCENE_HOVER, (2, 2, 4, 1), 8, 8, 1.0 / 60.0, 4, 4096,
                    description="C1 hover: 1 sphere over a static ground box"),
    "stack": Config("stack", SCENE_STACK, (9, 9, 32, 1), 8, 8, 1.0 / 60.0, 4, 16384,
                    description="C2 box stack: 8 unit boxes on a static ground box"),
    "chain": Config("chain", SCENE_CHAIN, (12, 12, 32, 10), 8, 8, 1.0 / 120.0, 2, 16384,
                    description="C3 chain: 10 capsules, weld + 9 revolutes (limits, springs, motors)"),
    "pile": Config("pile", SCENE_PILE, (37, 37, 128, 1), 8, 8, 1.0 / 60.0, 4, 65536, steps=240,
                   description="C4 pile: 16 boxes + 16 spheres between 4 walls"),
    # capacity-edge variants used by the tests: default capacities (body state
    # outside shared memory) and a contact capacity the stack overflows
    "default": Config("default", SCENE_PILE, (80, 128, 128, 32), 2, 2, 1.0 / 60.0, 4, 1024,
                      description="pile scene at the reference's default capacities"),
    "bounce": Config("bounce", SCENE_BOUNCE, (9, 9, 32, 1), 8, 8, 1.0 / 60.0, 4, 1024,
                     description="spheres and boxes with restitution and rolling resistance (parity coverage)"),
    "capsule": Config("capsule", SCENE_CAPSULE, (17, 17, 64, 1), 8, 8, 1.0 / 60.0, 4, 1024,
                      description="capsules and spheres falling into a walled bin (sphere-capsule and "
                                  "capsule-capsule manifolds)"),
    # the reference's alternative step modes (B3_INTERLEAVE_CONTACTS,
    # B3_SKIP_RESTITUTION) on the same scenes
    "stackil": Config("stackil", SCENE_STACK, (9, 9, 32, 1), 8, 8, 1.0 / 60.0, 4, 16384,
                      flags=STEP_INTERLEAVE_CONTACTS, description="stack, contacts interleaved with 8 iterations"),
    "chainil": Config("chainil", SCENE_CHAIN, (12, 12, 32, 10), 8, 8, 1.0 / 120.0, 2, 1024,
                      flags=STEP_INTERLEAVE_CONTACTS, description="chain, contacts interleaved with the joints"),
    "bouncenr": Config("bouncenr", SCENE_BOUNCE, (9, 9, 32, 1), 8, 8, 1.0 / 60.0, 4, 1024,
                       flags=STEP_SKIP_RESTITUTION, description="bounce without the restitution pass"),
    "bounceilnr": Config("bounceilnr", SCENE_BOUNCE, (9, 9, 32, 1), 8, 8, 1.0 / 60.0, 4, 1024,
                         flags=STEP_INTERLEAVE_CONTACTS | STEP_SKIP_RESTITUTION,
                         description="bounce, both modes"),
    "chainart": Config("chainart", SCENE_CHAIN, (12, 12, 32, 10), 8, 8, 1.0 / 120.0, 2, 1024,
                       description="chain with the articulated contact response (B3_ART_CONTACTS=1; "
                                   "per-thread step only)"),
    "hoveruf": Config("hoveruf", SCENE_HOVER, (2, 2, 4, 1), 8, 8, 1.0 / 60.0, 4, 1024,
                      description="hover with the per-substep force hook of scenes/b3_test_forces.h "
                                  "(B3_USER_FORCES; per-thread step only)"),
    "stacksmall": Config("stacksmall", SCENE_STACK, (9, 9, 4, 1), 2, 2, 1.0 / 60.0, 4, 1024,
                         description="stack scene with 4 contact slots (overflow path)"),
    "scaleout": Config("stack", SCENE_STACK, (9, 9, 32, 1), 8, 8, 1.0 / 60.0, 4, 1048576,
                       reset_fraction=0.01,
                       description="C5 scale-out: C2 worlds, 1% reset per step from snapshots"),
}
