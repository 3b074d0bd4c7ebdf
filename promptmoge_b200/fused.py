"""Fused multi-frame scene (benchmark configuration 5): one voxel grid back-projected from many camera poses, sharded over
GPUs by Morton (Z-order) ranges, with a one-voxel halo exchange before every submanifold conv.

The reference refines one frame at a time (moge/model/v3.py:305-344 voxelises one point map, one voxel per pixel);
the fused world-space grid is an extension of the benchmark with no reference counterpart.  What it keeps from the
reference is the operator: every layer is the int8 submanifold 3x3x3 conv of the refiner (submanifold_conv,
promptmoge/_fallback/flex_gemm/_core.py:399-441, under the QAT quantisers of moge/model/modules/qat.py:40-115), with
the reference's tap order and neighbour rule, so a sharded run must equal a single-device run over the whole grid
bit for bit, voxel by voxel.

Sharding.  Voxels are sorted by their Morton code; rank r of P owns the contiguous code range [lo_r, hi_r) (balanced
by voxel count), which in that order is the contiguous row range of a global index.  Each rank builds the neighbour
map of its own rows over the global voxel set, so a neighbour index outside [lo_r, hi_r) names the owner directly
(the rank whose range contains it).  The halo -- those outside rows, each listed once, sorted -- is appended after the
owned rows in a rank-local row space; before every conv the owners send the halo rows' int8 features with one
all-to-all (NCCL over NVLink on GPUs, gloo in the CPU tests).  Compute never crosses ranks; only int8 rows do.
"""
from __future__ import annotations

import math

import numpy as np
import torch

MORTON_BITS = 21


def _spread3(v: torch.Tensor) -> torch.Tensor:
    """Spread the low 21 bits of v (int64) so bit i lands at bit 3 i."""
    v = v & 0x1FFFFF
    v = (v | (v << 32)) & 0x1F00000000FFFF
    v = (v | (v << 16)) & 0x1F0000FF0000FF
    v = (v | (v << 8)) & 0x100F00F00F00F00F
    v = (v | (v << 4)) & 0x10C30C30C30C30C3
    v = (v | (v << 2)) & 0x1249249249249249
    return v


def _compact3(v: torch.Tensor) -> torch.Tensor:
    v = v & 0x1249249249249249
    v = (v | (v >> 2)) & 0x10C30C30C30C30C3
    v = (v | (v >> 4)) & 0x100F00F00F00F00F
    v = (v | (v >> 8)) & 0x1F0000FF0000FF
    v = (v | (v >> 16)) & 0x1F00000000FFFF
    v = (v | (v >> 32)) & 0x1FFFFF
    return v


def morton3(x: torch.Tensor, y: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
    """63-bit Morton code of non-negative 21-bit integer coordinates (x in the lowest bit of each triple)."""
    return _spread3(x.to(torch.int64)) | (_spread3(y.to(torch.int64)) << 1) | (_spread3(z.to(torch.int64)) << 2)


def demorton3(code: torch.Tensor):
    return _compact3(code), _compact3(code >> 1), _compact3(code >> 2)


# --------------------------------------------------------------------------------------------------------------- #
# Scene
# --------------------------------------------------------------------------------------------------------------- #

def _rotation(yaw: float, pitch: float) -> np.ndarray:
    """Camera-to-world rotation (camera x right, y down, z forward; world z up)."""
    base = np.array([[0.0, 0.0, 1.0], [-1.0, 0.0, 0.0], [0.0, -1.0, 0.0]])
    cy, sy = math.cos(yaw), math.sin(yaw)
    cp, sp = math.cos(pitch), math.sin(pitch)
    rz = np.array([[cy, -sy, 0], [sy, cy, 0], [0, 0, 1.0]])
    ry = np.array([[cp, 0, sp], [0, 1.0, 0], [-sp, 0, cp]])
    return rz @ ry @ base


def _raycast(origin: torch.Tensor, dirs: torch.Tensor, boxes: torch.Tensor, spheres: torch.Tensor,
             room: torch.Tensor) -> torch.Tensor:
    """Nearest hit parameter along each direction inside an axis-aligned room with boxes [n,2,3] and spheres
    [m,4] (centre, radius)."""
    inv = 1.0 / torch.where(dirs.abs() < 1e-12, torch.full_like(dirs, 1e-12), dirs)
    t = torch.maximum((room[0] - origin) * inv, (room[1] - origin) * inv).min(dim=1).values
    for lo, hi in boxes:
        a = (lo - origin) * inv
        b = (hi - origin) * inv
        tn = torch.minimum(a, b).max(dim=1).values
        tf = torch.maximum(a, b).min(dim=1).values
        hit = (tn <= tf) & (tn > 1e-3)
        t = torch.where(hit & (tn < t), tn, t)
    for s in spheres:
        oc = origin - s[:3]
        qa = (dirs * dirs).sum(dim=1)
        qb = 2.0 * (dirs @ oc)
        qc = float(oc @ oc) - float(s[3]) ** 2
        disc = qb * qb - 4 * qa * qc
        ok = disc > 0
        sq = torch.sqrt(torch.where(ok, disc, torch.zeros_like(disc)))
        tn = (-qb - sq) / (2 * qa)
        hit = ok & (tn > 1e-3)
        t = torch.where(hit & (tn < t), tn, t)
    return t


def make_fused_scene(seed: int, n_poses: int = 200, H: int = 480, W: int = 640, voxel: float = 0.01,
                     room_size=(12.0, 12.0, 3.0), device: str | torch.device = "cpu", chunk: int = 16):
    """Voxels (b = 0, x, y, z) int32 [M, 4] of one synthetic room seen from `n_poses` camera poses along a seeded random
    walk, back-projected with 1 %-of-depth noise into a `voxel`-metre grid, unique and sorted by Morton code.

    Room: `room_size` metres with one axis-aligned box per 3.6 m^2 of floor (40 in the 12 x 12 m room; 60 % standing
    on the floor) and one sphere per 18 m^2; pinhole camera fx = fy = 0.8 W at 1.2-1.8 m height, 0.15 m steps with a
    drifting heading.  Returns (coords, info)."""
    rng = np.random.default_rng(seed)
    dev = torch.device(device)
    room = np.array([[0.0, 0.0, 0.0], list(room_size)])
    area = room_size[0] * room_size[1]
    n_boxes, n_spheres = max(2, round(area / 3.6)), max(1, round(area / 18.0))
    boxes = []
    while len(boxes) < n_boxes:
        size = rng.uniform([0.3, 0.3, 0.3], [1.6, 1.6, 2.0])
        lo = rng.uniform(room[0], room[1] - size)
        if rng.random() < 0.6:
            lo[2] = 0.0
        boxes.append((lo, lo + size))
    spheres = []
    while len(spheres) < n_spheres:
        r = float(rng.uniform(0.2, 0.6))
        c = rng.uniform(room[0] + r, room[1] - r)
        spheres.append(np.concatenate([c, [r]]))

    def free(p):
        return all(not (np.all(p > lo - 0.3) and np.all(p < hi + 0.3)) for lo, hi in boxes) and \
            all(np.linalg.norm(p - s[:3]) > s[3] + 0.3 for s in spheres)

    def random_free():
        for _ in range(2000):
            p = np.array([rng.uniform(0.5, room_size[0] - 0.5), rng.uniform(0.5, room_size[1] - 0.5), 1.5])
            if free(p):
                return p
        return np.array([room_size[0] / 2, room_size[1] / 2, 1.5])   # crowded room: walk through furniture

    pos = random_free()
    heading = rng.uniform(-math.pi, math.pi)
    poses = []
    blocked = 0
    while len(poses) < n_poses:
        heading += rng.normal(0.0, 0.3)
        step = 0.15 * np.array([math.cos(heading), math.sin(heading), 0.0])
        cand = pos + step
        cand[2] = float(np.clip(cand[2] + rng.normal(0.0, 0.05), 1.2, 1.8))
        inside = 0.5 < cand[0] < room_size[0] - 0.5 and 0.5 < cand[1] < room_size[1] - 0.5
        if not inside or (blocked < 20 and not free(cand)):
            heading += math.pi / 2 + rng.uniform(0, math.pi)
            blocked += 1
            if blocked >= 40:                                  # boxed in: restart the walk elsewhere
                pos, blocked = random_free(), 0
            continue
        blocked = 0
        pos = cand
        poses.append((pos.copy(), _rotation(heading + rng.normal(0.0, 0.2), rng.uniform(-0.3, 0.3))))

    dt = torch.float32
    t_room = torch.tensor(room, dtype=dt, device=dev)
    t_boxes = torch.tensor(np.array([[lo, hi] for lo, hi in boxes]), dtype=dt, device=dev)
    t_spheres = torch.tensor(np.array(spheres), dtype=dt, device=dev)
    fx = 0.8 * W
    v, u = torch.meshgrid(torch.arange(H, dtype=dt, device=dev) + 0.5, torch.arange(W, dtype=dt, device=dev) + 0.5,
                          indexing="ij")
    d_cam = torch.stack([(u - W / 2.0) / fx, (v - H / 2.0) / fx, torch.ones_like(u)], dim=-1).reshape(-1, 3)
    noise_gen = torch.Generator(device=dev).manual_seed(seed)
    limit = (1 << MORTON_BITS) - 1
    codes = []
    pending = []
    for i, (o, R) in enumerate(poses):
        origin = torch.tensor(o, dtype=dt, device=dev)
        dirs = d_cam @ torch.tensor(R.T, dtype=dt, device=dev)
        t = _raycast(origin, dirs, t_boxes, t_spheres, t_room)
        t = t * (1.0 + 0.01 * torch.randn(t.shape, generator=noise_gen, device=dev, dtype=dt))
        p = origin + t[:, None] * dirs
        q = torch.floor(p / voxel).to(torch.int64).clamp(0, limit)
        pending.append(morton3(q[:, 0], q[:, 1], q[:, 2]))
        if len(pending) == chunk or i == len(poses) - 1:
            codes.append(torch.unique(torch.cat(pending)))
            pending = []
    code = torch.unique(torch.cat(codes))                 # sorted ascending = Morton order
    x, y, z = demorton3(code)
    coords = torch.stack([torch.zeros_like(x), x, y, z], dim=1).to(torch.int32)
    info = dict(seed=seed, poses=n_poses, H=H, W=W, voxel=voxel, room=list(room_size), voxels=int(coords.shape[0]))
    return coords, info


# --------------------------------------------------------------------------------------------------------------- #
# Sharding and halo exchange
# --------------------------------------------------------------------------------------------------------------- #

def shard_bounds(M: int, world: int):
    """Contiguous, count-balanced row ranges of the Morton-sorted voxels: [(lo, hi)] per rank."""
    cuts = [(M * r) // world for r in range(world + 1)]
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def tile_mask_of(nmap_tm: torch.Tensor) -> torch.Tensor:
    """Per 32-row group: OR of the occupied taps of a tap-major [27, M] map (int32 view of the uint32 words, one spare
    word as the kernels' masks have)."""
    M = nmap_tm.shape[1]
    G = (M + 31) // 32
    pres = torch.zeros((27, G * 32), dtype=torch.bool, device=nmap_tm.device)
    pres[:, :M] = nmap_tm >= 0
    anyg = pres.view(27, G, 32).any(dim=2).to(torch.int64)                       # [27, G]
    bits = (anyg << torch.arange(27, device=nmap_tm.device, dtype=torch.int64)[:, None]).sum(dim=0)
    out = torch.zeros(G + 1, dtype=torch.int64, device=nmap_tm.device)
    out[:G] = bits
    return out.to(torch.int32)


class ShardPlan:
    """Rank-local view of a Morton-sharded voxel set.

    `nmap_owned` is the tap-major [27, n_own] neighbour map of this rank's rows over the GLOBAL voxel set (global
    indices, -1 absent), as any of the library's neighbour-map builders give it for rows lo..hi.  The plan remaps it
    into the local row space [owned rows | halo rows] and sets up the exchange: which owned rows each peer needs
    (`send_idx`, grouped by peer) and how many rows arrive from each (`recv_splits`).  Collectives (two all-to-alls)
    run on `group`; every rank of the group must build its plan at the same time."""

    def __init__(self, nmap_owned: torch.Tensor, bounds, rank: int, group=None, peers_halo=None):
        """`peers_halo` (every rank's halo ids, in rank order) builds the send lists without collectives: the
        single-process emulation of several ranks that `exchange_in_process` runs."""
        import torch.distributed as dist
        self.rank = rank
        self.world = len(bounds)
        self.lo, self.hi = bounds[rank]
        self.n_own = self.hi - self.lo
        dev = nmap_owned.device
        outside = (nmap_owned >= 0) & ((nmap_owned < self.lo) | (nmap_owned >= self.hi))
        halo = torch.unique(nmap_owned[outside])                      # sorted global ids = grouped by owner
        self.halo = halo
        self.n_halo = int(halo.numel())
        # local nmap: owned -> id - lo, halo -> n_own + position, absent stays -1
        local = nmap_owned.clone()
        inside = (nmap_owned >= self.lo) & (nmap_owned < self.hi)
        local[inside] = nmap_owned[inside] - self.lo
        if self.n_halo:
            local[outside] = (self.n_own + torch.searchsorted(halo, nmap_owned[outside])).to(local.dtype)
        self.nmap = local.contiguous()
        self.mask = tile_mask_of(self.nmap)
        # owners of the halo rows and the exchange lists
        his = torch.tensor([b[1] for b in bounds], dtype=torch.int64, device=dev)
        owner = torch.searchsorted(his, halo.to(torch.int64), right=True) if self.n_halo else halo.to(torch.int64)
        recv_counts = torch.bincount(owner, minlength=self.world) if self.n_halo else \
            torch.zeros(self.world, dtype=torch.int64, device=dev)
        self.recv_splits = [int(c) for c in recv_counts.tolist()]
        if peers_halo is not None:
            parts = [h[(h >= self.lo) & (h < self.hi)] for h in peers_halo]
            self.send_splits = [int(x.numel()) for x in parts]
            wanted = torch.cat(parts) if parts else halo[:0]
        else:
            send_counts = torch.empty_like(recv_counts)
            if self.world > 1:
                dist.all_to_all_single(send_counts, recv_counts, group=group)
            else:
                send_counts.copy_(recv_counts)
            self.send_splits = [int(c) for c in send_counts.tolist()]
            wanted = torch.empty(sum(self.send_splits), dtype=halo.dtype, device=dev)
            if self.world > 1:
                dist.all_to_all_single(wanted, halo.contiguous(), self.send_splits, self.recv_splits, group=group)
            else:
                wanted.copy_(halo)
        if wanted.numel() and (int(wanted.min()) < self.lo or int(wanted.max()) >= self.hi):
            raise RuntimeError("halo request outside this rank's range")
        self.send_idx = (wanted.to(torch.int64) - self.lo).contiguous()
        self.group = group

    def local_buffer(self, C: int, dtype=torch.int8) -> torch.Tensor:
        """[n_own + n_halo, C] rows: owned first, halo rows after (filled by `exchange`)."""
        return torch.empty((self.n_own + self.n_halo, C), dtype=dtype, device=self.nmap.device)

    def exchange(self, buf: torch.Tensor) -> torch.Tensor:
        """Fill the halo rows of `buf` from their owners (one all-to-all of int8 rows)."""
        import torch.distributed as dist
        if self.world == 1 or (not self.n_halo and not self.send_idx.numel()):
            return buf
        send = buf.index_select(0, self.send_idx)
        dist.all_to_all_single(buf[self.n_own:], send, self.recv_splits, self.send_splits, group=self.group)
        return buf

    def halo_bytes(self, C: int) -> int:
        """int8 bytes this rank receives per conv layer."""
        return self.n_halo * C


def halo_ids(nmap_owned: torch.Tensor, lo: int, hi: int) -> torch.Tensor:
    """Global ids outside [lo, hi) that the owned rows' neighbour map references, sorted, each once."""
    outside = (nmap_owned >= 0) & ((nmap_owned < lo) | (nmap_owned >= hi))
    return torch.unique(nmap_owned[outside])


def plans_in_process(nmap_tm: torch.Tensor, bounds):
    """Plans of every rank built in one process from the global tap-major map (no collectives)."""
    halos = [halo_ids(nmap_tm[:, lo:hi], lo, hi) for lo, hi in bounds]
    return [ShardPlan(nmap_tm[:, lo:hi].contiguous(), bounds, r, peers_halo=halos) for r, (lo, hi) in enumerate(bounds)]


def exchange_in_process(plans, bufs):
    """The all-to-all of `ShardPlan.exchange` for ranks emulated in one process (buffers of all ranks)."""
    for r, pr in enumerate(plans):
        off = pr.n_own
        for p, pp in enumerate(plans):
            n = pr.recv_splits[p]
            if n == 0:
                continue
            s0 = sum(pp.send_splits[:r])
            bufs[r][off:off + n] = bufs[p].index_select(0, pp.send_idx[s0:s0 + n])
            off += n


def run_layers(plan: ShardPlan, q_own: torch.Tensor, layers, conv) -> torch.Tensor:
    """A stack of int8 submanifold convs over the sharded voxels: before each layer the halo rows are exchanged, then
    `conv(q_local, nmap, mask, layer)` returns the next int8 features of the owned rows."""
    buf = plan.local_buffer(q_own.shape[1], q_own.dtype)
    buf[:plan.n_own] = q_own
    for layer in layers:
        plan.exchange(buf)
        out = conv(buf, plan.nmap, plan.mask, layer)
        buf[:plan.n_own] = out
    return buf[:plan.n_own].clone()


def gpu_conv(q_local, nmap, mask, layer):
    """The product conv of a layer: tcgen05 int8 submanifold conv with the fused SiLU + requantise epilogue."""
    from . import ops
    w, ws, b, sa, s_out = layer
    return ops.spconv_i8(q_local, nmap, mask, w, ws, b, sa, ops.EPI_SILU_Q8, s_out, rows=nmap.shape[1])


def random_layers(n: int, C: int, seed: int, device):
    """Seeded int8 weights [27, C, C], per-channel scales, biases and activation scales for `n` layers."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    layers = []
    for _ in range(n):
        w = torch.randint(-127, 128, (27, C, C), generator=g, dtype=torch.int8)
        ws = torch.rand(C, generator=g) * 4e-4 + 1e-4
        b = torch.randn(C, generator=g) * 0.1
        layers.append((w.to(device), ws.to(device), b.to(device), 0.05, 0.04))
    return layers
