"""Synthetic f32 volumes of the benchmark configurations, generated on the GPU.

Every generator is a pure function of the global node index (i, j, k) and a
seed, evaluated plane by plane, so a z-slab [k0, k1) generated on one rank
holds exactly the bytes of the same planes of the whole volume.  Random
parameters (blob centres, frequencies, phases) come from numpy's PCG64 with
the given seed; per-node noise comes from a counter-based integer hash of the
node index, not from a stateful generator.

Configurations (nodes per axis; unit spacing, origin 0):
  sphere   C1  64^3: |idx - 31.5| - 20, isovalue 0
  gyroid   C2  256^3: sin x cos y + sin y cos z + sin z cos x with
               x,y,z = 2*pi*4*idx/n, plus N(0, 0.01) noise, isovalue 0
  sines    C3  512^3: sum of 8 a*sin(2*pi*k.idx/n + phi), k in [1,16]^3
               integers, phi U(0, 2pi), a U(0.5, 1), isovalue 0.25
  blobs    C4  1024^3: sum of 32 w*exp(-|idx-c|^2 / (2 s^2)), c U(0,n)^3,
               s U(20,80) * n/1024, w U(0.5,1.5), isovalue 0.5
  noise    C5  2048x2048x1024: 4-octave value noise, lattice values U(-1,1),
               trilinear, gain 0.5, frequency x2 per octave, base lattice
               period 128 nodes, isovalues {-0.3, 0, 0.3, 0.6}
"""

import math

import numpy as np
import torch

CONFIGS = {
    "sphere": {"shape": (64, 64, 64), "isovalues": [0.0], "seed": 0},
    "gyroid": {"shape": (256, 256, 256), "isovalues": [0.0], "seed": 2},
    "sines": {"shape": (512, 512, 512), "isovalues": [0.25], "seed": 3},
    "blobs": {"shape": (1024, 1024, 1024), "isovalues": [0.5], "seed": 4},
    "noise": {"shape": (2048, 2048, 1024), "isovalues": [-0.3, 0.0, 0.3, 0.6], "seed": 5},
}

_M64 = (1 << 64) - 1


def _to_i64(x):
    x &= _M64
    return x - (1 << 64) if x >= 1 << 63 else x


def _hash_u32(idx, seed):
    """Counter-based hash of int64 node indices -> uint32 values (int64 tensor).

    A 64-bit multiply-xorshift mixer; int64 arithmetic wraps in torch, and
    the final value is the high 32 bits.
    """
    x = idx * _to_i64(0x9E3779B97F4A7C15) + _to_i64((seed * 0xD1B54A32D192ED03) & _M64)
    x = x ^ ((x >> 31) & 0x1FFFFFFFF)
    x = x * _to_i64(0xBF58476D1CE4E5B9)
    x = x ^ ((x >> 27) & 0x1FFFFFFFFF)
    x = x * _to_i64(0x94D049BB133111EB)
    x = x ^ ((x >> 31) & 0x1FFFFFFFF)
    return (x >> 32) & 0xFFFFFFFF


def _uniform(idx, seed):
    """U(0,1) in (0, 1], float64, from the hash."""
    return (_hash_u32(idx, seed).to(torch.float64) + 1.0) / 4294967296.0


def _normal(idx, seed):
    """N(0,1) by Box-Muller from two hashed uniforms, float64."""
    u1 = _uniform(idx, seed)
    u2 = _uniform(idx, seed ^ 0x5bd1e995)
    return torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * math.pi * u2)


def _plane_coords(nx, ny, device, dtype):
    j = torch.arange(ny, device=device, dtype=dtype).view(ny, 1)
    i = torch.arange(nx, device=device, dtype=dtype).view(1, nx)
    return i, j


def generate(name, shape=None, k0=0, k1=None, seed=None, device=None, out=None,
             planes_per_step=None):
    """Planes [k0, k1) of configuration `name` as a flat f32 CUDA tensor.

    shape = (nx_nodes, ny_nodes, nz_nodes), defaulting to the configuration's.
    The result has (k1-k0)*ny*nx values, i fastest.
    """
    cfg = CONFIGS[name]
    nx, ny, nz = shape or cfg["shape"]
    k1 = nz if k1 is None else k1
    if not (0 <= k0 <= k1 <= nz):
        raise ValueError(f"plane range [{k0}, {k1}) outside 0..{nz}")
    seed = cfg["seed"] if seed is None else seed
    device = device or torch.device("cuda", torch.cuda.current_device())
    nplanes = k1 - k0
    if out is None:
        out = torch.empty(nplanes * ny * nx, dtype=torch.float32, device=device)
    fn = {"sphere": _sphere, "gyroid": _gyroid, "sines": _sines, "blobs": _blobs,
          "noise": _noise}[name]
    params = _params(name, (nx, ny, nz), seed)
    step = planes_per_step or max(1, (1 << 24) // max(1, nx * ny))
    view = out.view(nplanes, ny, nx)
    for ka in range(k0, k1, step):
        kb = min(k1, ka + step)
        view[ka - k0:kb - k0] = fn((nx, ny, nz), ka, kb, params, device)
    return out


def _params(name, shape, seed):
    rng = np.random.default_rng(seed)
    nx, ny, nz = shape
    if name == "sines":
        return {"k": rng.integers(1, 17, size=(8, 3)), "phi": rng.uniform(0, 2 * np.pi, 8),
                "a": rng.uniform(0.5, 1.0, 8)}
    if name == "blobs":
        scale = max(nx, ny, nz) / 1024.0
        return {"c": rng.uniform(0, 1, size=(32, 3)) * np.array([nx, ny, nz]),
                "s": rng.uniform(20, 80, 32) * scale, "w": rng.uniform(0.5, 1.5, 32)}
    if name == "noise":
        return {"seed": seed, "period": 128, "octaves": 4}
    return {"seed": seed}


def _sphere(shape, ka, kb, p, device):
    nx, ny, _ = shape
    i, j = _plane_coords(nx, ny, device, torch.float64)
    k = torch.arange(ka, kb, device=device, dtype=torch.float64).view(-1, 1, 1)
    r = torch.sqrt((i - 31.5) ** 2 + (j - 31.5) ** 2 + (k - 31.5) ** 2)
    return (r - 20.0).to(torch.float32)


def _gyroid(shape, ka, kb, p, device):
    nx, ny, nz = shape
    i, j = _plane_coords(nx, ny, device, torch.float64)
    k = torch.arange(ka, kb, device=device, dtype=torch.float64).view(-1, 1, 1)
    x = 2 * math.pi * 4 * i / nx
    y = 2 * math.pi * 4 * j / ny
    z = 2 * math.pi * 4 * k / nz
    v = torch.sin(x) * torch.cos(y) + torch.sin(y) * torch.cos(z) + torch.sin(z) * torch.cos(x)
    idx = (torch.arange(ka, kb, device=device, dtype=torch.int64).view(-1, 1, 1) * ny
           + torch.arange(ny, device=device, dtype=torch.int64).view(1, ny, 1)) * nx \
        + torch.arange(nx, device=device, dtype=torch.int64).view(1, 1, nx)
    v = v + 0.01 * _normal(idx, p["seed"])
    return v.to(torch.float32)


def _sines(shape, ka, kb, p, device):
    nx, ny, nz = shape
    i, j = _plane_coords(nx, ny, device, torch.float64)
    k = torch.arange(ka, kb, device=device, dtype=torch.float64).view(-1, 1, 1)
    v = torch.zeros((kb - ka, ny, nx), dtype=torch.float64, device=device)
    for m in range(8):
        kx, ky, kz = (int(t) for t in p["k"][m])
        ph = 2 * math.pi * (kx * i / nx + ky * j / ny + kz * k / nz) + float(p["phi"][m])
        v += float(p["a"][m]) * torch.sin(ph)
    return v.to(torch.float32)


def _blobs(shape, ka, kb, p, device):
    nx, ny, _ = shape
    i, j = _plane_coords(nx, ny, device, torch.float32)
    k = torch.arange(ka, kb, device=device, dtype=torch.float32).view(-1, 1, 1)
    v = torch.zeros((kb - ka, ny, nx), dtype=torch.float32, device=device)
    for m in range(32):
        cx, cy, cz = (float(t) for t in p["c"][m])
        inv = -1.0 / (2.0 * float(p["s"][m]) ** 2)
        dz2 = (k - cz) ** 2
        dxy2 = (i - cx) ** 2 + (j - cy) ** 2
        v += float(p["w"][m]) * torch.exp((dxy2 + dz2) * inv)
    return v


def _lattice(ix, iy, iz, seed, per):
    """Lattice value U(-1,1) at integer lattice points (periodic `per`)."""
    idx = ((iz % per[2]) * per[1] + (iy % per[1])) * per[0] + (ix % per[0])
    return 2.0 * _uniform(idx, seed) - 1.0


def _noise(shape, ka, kb, p, device):
    nx, ny, nz = shape
    v = torch.zeros((kb - ka, ny, nx), dtype=torch.float64, device=device)
    i = torch.arange(nx, device=device, dtype=torch.float64).view(1, 1, nx)
    j = torch.arange(ny, device=device, dtype=torch.float64).view(1, ny, 1)
    k = torch.arange(ka, kb, device=device, dtype=torch.float64).view(-1, 1, 1)
    amp = 1.0
    period = float(p["period"])
    for o in range(p["octaves"]):
        fx, fy, fz = i / period, j / period, k / period
        x0, y0, z0 = torch.floor(fx), torch.floor(fy), torch.floor(fz)
        tx, ty, tz = fx - x0, fy - y0, fz - z0
        x0, y0, z0 = x0.to(torch.int64), y0.to(torch.int64), z0.to(torch.int64)
        per = (max(1, int(math.ceil(nx / period))) + 1, max(1, int(math.ceil(ny / period))) + 1,
               max(1, int(math.ceil(nz / period))) + 1)
        s = p["seed"] * 131 + o
        acc = torch.zeros_like(v)
        for dz in (0, 1):
            wz = tz if dz else 1 - tz
            for dy in (0, 1):
                wy = ty if dy else 1 - ty
                for dx in (0, 1):
                    wx = tx if dx else 1 - tx
                    acc += wx * wy * wz * _lattice(x0 + dx, y0 + dy, z0 + dz, s, per)
        v += amp * acc
        amp *= 0.5
        period /= 2.0
    return v.to(torch.float32)
