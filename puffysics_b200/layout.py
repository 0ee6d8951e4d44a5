"""numpy mirror of the B3World memory layout (include/puffysics_b200.h).

The layout is the reference's AoS struct for given capacities
(reference src/puffysics/02_types.inl:55-332): a 68-byte header, then
bodies[B] (200 B), shapes[S] (88 B, 8-byte aligned), contacts[C] (476 B),
joints[J] (460 B), padded to 8 bytes.  Used by the host side to decode and
inspect worlds (tests, benchmark observations); the kernels decode the same
offsets at run time from the capacity signature.
"""
import numpy as np

f4 = np.float32
i4 = np.int32
u4 = np.uint32
u8 = np.uint64

VEC3 = (f4, (3,))
QUAT = (f4, (4,))          # x, y, z, s
MAT3 = (f4, (3, 3))        # columns cx, cy, cz
SOFT = (f4, (3,))          # bias_rate, mass_scale, impulse_scale

BODY = np.dtype([
    ("position", VEC3), ("rotation", QUAT), ("center", VEC3), ("local_center", VEC3),
    ("lin_vel", VEC3), ("ang_vel", VEC3), ("force", VEC3), ("torque", VEC3),
    ("delta_pos", VEC3), ("delta_rot", QUAT), ("inv_mass", f4), ("inv_inertia", VEC3),
    ("inv_i_world", MAT3), ("linear_damping", f4), ("angular_damping", f4), ("gravity_scale", f4),
    ("type", i4), ("flags", u4),
])
SHAPE = np.dtype({
    "names": ["body", "type", "local_pos", "local_rot", "radius", "half", "friction", "restitution",
              "rolling", "density", "category", "mask"],
    "formats": [i4, i4, VEC3, QUAT, f4, VEC3, f4, f4, f4, f4, u8, u8],
    "offsets": [0, 4, 8, 20, 36, 40, 52, 56, 60, 64, 72, 80],
    "itemsize": 88,
})
POINT = np.dtype([
    ("r_a", VEC3), ("r_b", VEC3), ("base_sep", f4), ("rel_vel", f4), ("normal_impulse", f4),
    ("total_normal", f4), ("normal_mass", f4), ("lever", f4), ("feature", u4),
])
CONTACT = np.dtype([
    ("shape_a", i4), ("shape_b", i4), ("body_a", i4), ("body_b", i4), ("point_count", i4),
    ("static_contact", i4), ("normal", VEC3), ("tangent1", VEC3), ("tangent2", VEC3),
    ("points", POINT, (4,)), ("center_a", VEC3), ("center_b", VEC3), ("friction", f4),
    ("restitution", f4), ("rolling", f4), ("twist_mass", f4), ("twist_impulse", f4),
    ("friction_impulse", (f4, (2,))), ("rolling_impulse", VEC3), ("tangent_mass", (f4, (4,))),
    ("rolling_mass", MAT3), ("inv_mass_a", f4), ("inv_mass_b", f4), ("inv_i_a", MAT3),
    ("inv_i_b", MAT3), ("softness", SOFT),
])
JOINT = np.dtype([
    ("type", i4), ("body_a", i4), ("body_b", i4), ("collide_connected", i4), ("fixed_rotation", i4),
    ("local_anchor_a", VEC3), ("local_anchor_b", VEC3), ("local_rot_a", QUAT), ("local_rot_b", QUAT),
    ("constraint_hertz", f4), ("constraint_damping", f4), ("softness", SOFT),
    ("inv_mass_a", f4), ("inv_mass_b", f4), ("inv_i_a", MAT3), ("inv_i_b", MAT3),
    ("frame_p_a", VEC3), ("frame_p_b", VEC3), ("frame_q_a", QUAT), ("frame_q_b", QUAT),
    ("delta_center", VEC3), ("linear_impulse", VEC3), ("angular_impulse", VEC3), ("angular_mass", MAT3),
    ("linear_hertz", f4), ("linear_damping", f4), ("angular_hertz", f4), ("angular_damping", f4),
    ("linear_spring", SOFT), ("angular_spring", SOFT), ("perp_impulse", (f4, (2,))),
    ("spring_impulse", f4), ("motor_impulse", f4), ("lower_impulse", f4), ("upper_impulse", f4),
    ("hertz", f4), ("damping_ratio", f4), ("max_motor_torque", f4), ("motor_speed", f4),
    ("target_angle", f4), ("lower_angle", f4), ("upper_angle", f4), ("enable_spring", i4),
    ("enable_motor", i4), ("enable_limit", i4), ("rotation_axis", VEC3), ("perp_x", VEC3),
    ("perp_y", VEC3), ("axial_mass", f4), ("spring_softness", SOFT),
])
HEADER = np.dtype([
    ("gravity", VEC3), ("contact_hertz", f4), ("contact_damping", f4), ("contact_speed", f4),
    ("restitution_threshold", f4), ("max_linear_speed", f4), ("body_count", i4), ("shape_count", i4),
    ("contact_count", i4), ("joint_count", i4), ("body_overflow", i4), ("shape_overflow", i4),
    ("joint_overflow", i4), ("contact_overflow", i4), ("contacts_dropped", i4),
])
assert BODY.itemsize == 200 and SHAPE.itemsize == 88 and POINT.itemsize == 52
assert CONTACT.itemsize == 476 and JOINT.itemsize == 460 and HEADER.itemsize == 68


def signature(bodies, shapes, contacts, joints):
    return (bodies & 0xFFFF) | ((shapes & 0xFFFF) << 16) | ((contacts & 0xFFFF) << 32) | ((joints & 0xFFFF) << 48)


def caps_from_signature(sig):
    return tuple((sig >> s) & 0xFFFF for s in (0, 16, 32, 48))


def world_dtype(bodies, shapes, contacts, joints):
    """Structured dtype of one B3World with these capacities."""
    body_off = HEADER.itemsize
    shape_off = body_off + 200 * bodies
    shape_off = (shape_off + 7) & ~7
    contact_off = shape_off + 88 * shapes
    joint_off = contact_off + 476 * contacts
    size = (joint_off + 460 * joints + 7) & ~7
    names = list(HEADER.names) + ["bodies", "shapes", "contacts", "joints"]
    formats = [HEADER.fields[n][0] for n in HEADER.names] + [
        (BODY, (bodies,)), (SHAPE, (shapes,)), (CONTACT, (contacts,)), (JOINT, (joints,))]
    offsets = [HEADER.fields[n][1] for n in HEADER.names] + [body_off, shape_off, contact_off, joint_off]
    return np.dtype({"names": names, "formats": formats, "offsets": offsets, "itemsize": size})


def world_bytes(bodies, shapes, contacts, joints):
    return world_dtype(bodies, shapes, contacts, joints).itemsize


def view(raw, caps):
    """Structured view (count,) of a (count, world_bytes) uint8 array."""
    dt = world_dtype(*caps)
    raw = np.ascontiguousarray(raw)
    assert raw.shape[-1] == dt.itemsize, (raw.shape, dt.itemsize)
    return raw.view(dt).reshape(raw.shape[:-1])
