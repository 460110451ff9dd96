"""Seeded synthetic aux ray fields for the ray->pose solver tests.

A camera with rotation R (small random angles), normalised intrinsics (focal f,
principal point p) and centre C emits, for each point of the identity-plane grid the
solver uses (src/ray_pose.cpp:23-31), the world direction R @ ((x - p) / f, 1) and the
origin C; a fraction of points get random directions (outliers), all get small noise,
and confidences are uniform in [1, 3]."""
import numpy as np


def rot(a, b, c):
    ca, sa, cb, sb, cc, sc = np.cos(a), np.sin(a), np.cos(b), np.sin(b), np.cos(c), np.sin(c)
    Rx = np.array([[1, 0, 0], [0, ca, -sa], [0, sa, ca]])
    Ry = np.array([[cb, 0, sb], [0, 1, 0], [-sb, 0, cb]])
    Rz = np.array([[cc, -sc, 0], [sc, cc, 0], [0, 0, 1]])
    return Rz @ Ry @ Rx


def field(seed, Hy, Wx, outliers=0.2, noise=1e-3):
    """(ray [Hy][Wx][6] f32, conf [Hy][Wx] f32, truth dict)."""
    rng = np.random.default_rng(seed)
    f = rng.uniform(0.6, 1.6, 2)
    p = rng.uniform(-0.1, 0.1, 2)
    R = rot(*rng.uniform(-0.3, 0.3, 3))
    C = rng.uniform(-1, 1, 3)
    dx, dy = 1.0 / Wx, 1.0 / Hy
    gx = np.linspace(dx, 2 - dx, Wx) - 1.0
    gy = np.linspace(dy, 2 - dy, Hy) - 1.0
    X, Y = np.meshgrid(gx, gy)
    cam = np.stack([(X - p[0]) / f[0], (Y - p[1]) / f[1], np.ones_like(X)], -1)
    d = cam @ R.T
    bad = rng.random((Hy, Wx)) < outliers
    d[bad] = rng.standard_normal((int(bad.sum()), 3))
    d += rng.standard_normal(d.shape) * noise
    o = np.broadcast_to(C, d.shape) + rng.standard_normal(d.shape) * noise
    ray = np.concatenate([d, o], -1).astype(np.float32)
    conf = rng.uniform(1.0, 3.0, (Hy, Wx)).astype(np.float32)
    return ray, conf, {"f": f, "p": p, "R": R, "C": C}
