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


def scene_layout(seed: int, n_poses: int = 200, room_size=(12.0, 12.0, 3.0)):
    """The seeded room and camera walk of a fused scene: (room [2,3], boxes [(lo, hi)], spheres [[c, r]], poses
    [(position, rotation)]).  Room: `room_size` metres with one axis-aligned box per 3.6 m^2 of floor (40 in the
    12 x 12 m room; 60 % standing on the floor) and one sphere per 18 m^2; camera at 1.2-1.8 m height, 0.15 m steps
    with a drifting heading.  Plain numpy from the seed: every rank derives the same layout."""
    rng = np.random.default_rng(seed)
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
    return room, boxes, spheres, poses


def scene_codes(seed: int, layout, pose_ids, H: int = 480, W: int = 640, voxel: float = 0.01,
                device: str | torch.device = "cpu", chunk: int = 16) -> torch.Tensor:
    """Sorted unique Morton codes (int64) of the voxels the poses `pose_ids` of `layout` back-project into: pinhole
    fx = fy = 0.8 W, analytic ray cast, 1 %-of-depth noise drawn from a generator seeded by (seed, pose index), so a
    pose gives the same voxels whichever rank casts it."""
    room, boxes, spheres, poses = layout
    dev = torch.device(device)
    dt = torch.float32
    t_room = torch.tensor(room, dtype=dt, device=dev)
    t_boxes = torch.tensor(np.array([[lo, hi] for lo, hi in boxes]), dtype=dt, device=dev)
    t_spheres = torch.tensor(np.array(spheres), dtype=dt, device=dev)
    fx = 0.8 * W
    v, u = torch.meshgrid(torch.arange(H, dtype=dt, device=dev) + 0.5, torch.arange(W, dtype=dt, device=dev) + 0.5,
                          indexing="ij")
    d_cam = torch.stack([(u - W / 2.0) / fx, (v - H / 2.0) / fx, torch.ones_like(u)], dim=-1).reshape(-1, 3)
    limit = (1 << MORTON_BITS) - 1
    codes, pending = [], []
    pose_ids = list(pose_ids)
    for n, i in enumerate(pose_ids):
        o, R = poses[i]
        origin = torch.tensor(o, dtype=dt, device=dev)
        dirs = d_cam @ torch.tensor(R.T, dtype=dt, device=dev)
        t = _raycast(origin, dirs, t_boxes, t_spheres, t_room)
        gen = torch.Generator(device=dev).manual_seed(seed * 1_000_003 + i)
        t = t * (1.0 + 0.01 * torch.randn(t.shape, generator=gen, device=dev, dtype=dt))
        p = origin + t[:, None] * dirs
        q = torch.floor(p / voxel).to(torch.int64).clamp(0, limit)
        pending.append(morton3(q[:, 0], q[:, 1], q[:, 2]))
        if len(pending) == chunk or n == len(pose_ids) - 1:
            codes.append(torch.unique(torch.cat(pending)))
            pending = []
    if not codes:
        return torch.empty(0, dtype=torch.int64, device=dev)
    return torch.unique(torch.cat(codes))                 # sorted ascending = Morton order


def coords_of_codes(code: torch.Tensor) -> torch.Tensor:
    """[M, 4] int32 (b = 0, x, y, z) of Morton codes."""
    x, y, z = demorton3(code)
    return torch.stack([torch.zeros_like(x), x, y, z], dim=1).to(torch.int32)


def make_fused_scene(seed: int, n_poses: int = 200, H: int = 480, W: int = 640, voxel: float = 0.01,
                     room_size=(12.0, 12.0, 3.0), device: str | torch.device = "cpu", chunk: int = 16):
    """Voxels (b = 0, x, y, z) int32 [M, 4] of one synthetic room (scene_layout) seen from `n_poses` camera poses,
    back-projected (scene_codes) into a `voxel`-metre grid, unique and sorted by Morton code.  Returns (coords, info)."""
    layout = scene_layout(seed, n_poses, room_size)
    code = scene_codes(seed, layout, range(n_poses), H, W, voxel, device, chunk)
    coords = coords_of_codes(code)
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
        self._split_boundary()

    @classmethod
    def from_parts(cls, nmap_local: torch.Tensor, n_own: int, n_halo: int, recv_splits, send_idx: torch.Tensor,
                   send_splits, rank: int, world: int, group=None) -> "ShardPlan":
        """A plan from an already local neighbour map (owned rows, indices in [owned | halo] row space) and the
        exchange lists, for a voxel set sharded without a global view (LevelShard)."""
        self = cls.__new__(cls)
        self.rank, self.world = rank, world
        self.lo, self.hi = 0, n_own
        self.n_own, self.n_halo = n_own, n_halo
        self.halo = None
        self.nmap = nmap_local.contiguous()
        self.mask = tile_mask_of(self.nmap)
        self.recv_splits = [int(c) for c in recv_splits]
        self.send_splits = [int(c) for c in send_splits]
        self.send_idx = send_idx.to(torch.int64).contiguous()
        self.group = group
        self._split_boundary()
        return self

    def _split_boundary(self):
        """Interior rows (every neighbour owned) and boundary rows (some neighbour in the halo), for the conv that
        overlaps the exchange: `perm` lists the owned rows interior first (each part in row order), `nmap_int` /
        `nmap_bnd` are the two parts' columns of the neighbour map (indices still in the [owned | halo] row space)."""
        bnd = (self.nmap >= self.n_own).any(dim=0) if self.n_own else torch.zeros(0, dtype=torch.bool,
                                                                                    device=self.nmap.device)
        inner = torch.nonzero(~bnd).flatten()
        edge = torch.nonzero(bnd).flatten()
        self.n_int = int(inner.numel())
        self.perm = torch.cat([inner, edge])
        self.nmap_int = self.nmap[:, inner].contiguous()
        self.nmap_bnd = self.nmap[:, edge].contiguous()
        self.mask_int = tile_mask_of(self.nmap_int)
        self.mask_bnd = tile_mask_of(self.nmap_bnd)

    def local_buffer(self, C: int, dtype=torch.int8) -> torch.Tensor:
        """[n_own + n_halo, C] rows: owned first, halo rows after (filled by `exchange`)."""
        return torch.empty((self.n_own + self.n_halo, C), dtype=dtype, device=self.nmap.device)

    def exchange(self, buf: torch.Tensor) -> torch.Tensor:
        """Fill the halo rows of `buf` from their owners (one all-to-all of int8 rows).  Every rank of the group takes
        part, also one that neither sends nor receives (a collective must be entered by all of them)."""
        import torch.distributed as dist
        if self.world == 1:
            return buf
        send = buf.index_select(0, self.send_idx)
        dist.all_to_all_single(buf[self.n_own:], send, self.recv_splits, self.send_splits, group=self.group)
        return buf

    def conv(self, buf: torch.Tensor, layer, conv, overlap: bool = False) -> None:
        """One conv layer in place on the owned rows of `buf`: exchange the halo rows, then
        `conv(q_local, nmap, mask, layer)`.  overlap: the interior rows' conv runs while the all-to-all is in flight
        (it reads owned rows only) and the boundary rows' conv after it lands; both parts write their rows back in
        row order, so the result equals the plain exchange-then-conv bit for bit."""
        import torch.distributed as dist
        if not (overlap and self.world > 1):
            self.exchange(buf)
            buf[:self.n_own] = conv(buf, self.nmap, self.mask, layer)
            return
        send = buf.index_select(0, self.send_idx)
        work = dist.all_to_all_single(buf[self.n_own:], send, self.recv_splits, self.send_splits, group=self.group,
                                      async_op=True)
        parts = []
        if self.n_int:
            parts.append(conv(buf, self.nmap_int, self.mask_int, layer))
        work.wait()
        if self.n_own - self.n_int:
            parts.append(conv(buf, self.nmap_bnd, self.mask_bnd, layer))
        if parts:                          # a rank may own no voxel of a level (it still took part in the exchange)
            buf[:self.n_own].index_copy_(0, self.perm, torch.cat(parts) if len(parts) > 1 else parts[0])

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


def run_layers(plan: ShardPlan, q_own: torch.Tensor, layers, conv, overlap: bool = False) -> torch.Tensor:
    """A stack of int8 submanifold convs over the sharded voxels: before each layer the halo rows are exchanged, then
    `conv(q_local, nmap, mask, layer)` returns the next int8 features of the owned rows (ShardPlan.conv)."""
    buf = plan.local_buffer(q_own.shape[1], q_own.dtype)
    buf[:plan.n_own] = q_own
    for layer in layers:
        plan.conv(buf, layer, conv, overlap)
    return buf[:plan.n_own].clone()


def gpu_conv(q_local, nmap, mask, layer):
    """The product conv of a layer: tcgen05 int8 submanifold conv with the fused SiLU + requantise epilogue."""
    from . import ops
    w, ws, b, sa, s_out = layer
    if nmap.shape[1] == 0:                 # no output rows (a rank that owns none of a level's voxels)
        return torch.empty((0, w.shape[1]), dtype=torch.int8, device=q_local.device)
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


# --------------------------------------------------------------------------------------------------------------- #
# Sharded structure without a global view: every rank back-projects its own poses, voxels go to the owners of their
# Morton code ranges (balanced per level), neighbours across a range boundary are looked up at their owner, and each
# coarser level is the set of parents (code >> 3) of the level below, with its own balanced ranges.
# --------------------------------------------------------------------------------------------------------------- #

LOCAL = "local"   # pass as `group` to run a sharded routine as the only rank (a single-device run), collectives off


def _world(group):
    import torch.distributed as dist
    if group is LOCAL or not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _alltoallv(send: torch.Tensor, send_counts, group):
    """Variable all-to-all of rows grouped by destination rank: (received rows grouped by source, counts)."""
    import torch.distributed as dist
    world, _ = _world(group)
    if world == 1:
        return send.clone(), [int(c) for c in send_counts]
    dev = send.device
    sc = torch.tensor([int(c) for c in send_counts], dtype=torch.int64, device=dev)
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc, group=group)
    recv_counts = [int(c) for c in rc.tolist()]
    recv = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype, device=dev)
    dist.all_to_all_single(recv, send.contiguous(), recv_counts, [int(c) for c in send_counts], group=group)
    return recv, recv_counts


def _owner_of(codes: torch.Tensor, splitters: torch.Tensor) -> torch.Tensor:
    """Rank whose code range [splitters[r], splitters[r + 1]) holds each code."""
    return torch.searchsorted(splitters[1:-1].contiguous(), codes, right=True)


CODE_END = (1 << 63) - 1      # end of the last code range (the all-ones 63-bit code, a voxel at 2^21 - 1 on every axis,
                              # is not used: scene coordinates stay far below it)


def morton_splitters(local_codes: torch.Tensor, group=None, samples: int = 1024, weights=None) -> torch.Tensor:
    """Code-range boundaries [world + 1] (int64) balancing the voxel counts (or the per-voxel `weights`, aligned with
    `local_codes`) over the ranks: every rank contributes `samples` codes at evenly spaced quantiles of the cumulative
    weight of its sorted codes, each carrying 1/samples of its total (one all-gather), and the ranges are cut at equal
    cumulative weight.  Codes several ranks back-project are counted once per rank here, which only perturbs the
    balance."""
    import torch.distributed as dist
    world, _ = _world(group)
    dev = local_codes.device
    if world == 1:
        return torch.tensor([0, CODE_END], dtype=torch.int64, device=dev)
    srt, order = torch.sort(local_codes)
    n = int(srt.numel())
    if n and weights is not None:
        cw = torch.cumsum(weights.to(torch.float64)[order], 0)
        tot = float(cw[-1])
        at = torch.arange(samples, device=dev, dtype=torch.float64) * (tot / samples)
        pick = srt[torch.searchsorted(cw, at, right=True).clamp(max=n - 1)]
    elif n:
        tot = float(n)
        pick = srt[(torch.arange(samples, device=dev) * n) // samples]
    else:
        tot = 0.0
        pick = torch.full((samples,), CODE_END, dtype=torch.int64, device=dev)
    meta = torch.tensor([tot], dtype=torch.float64, device=dev)
    picks = [torch.empty_like(pick) for _ in range(world)]
    metas = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(picks, pick, group=group)
    dist.all_gather(metas, meta, group=group)
    vals = torch.cat(picks)
    wts = torch.cat([torch.full((samples,), float(m.item()) / samples, dtype=torch.float64, device=dev)
                     for m in metas])
    order = torch.argsort(vals, stable=True)
    vals, cum = vals[order], torch.cumsum(wts[order], 0)
    total = float(cum[-1]) if cum.numel() else 0.0
    cuts = [0]
    for r in range(1, world):
        k = int(torch.searchsorted(cum, torch.tensor(total * r / world, dtype=torch.float64, device=dev)))
        cuts.append(max(int(vals[min(k, vals.numel() - 1)]), cuts[-1]))
    cuts.append(CODE_END)
    return torch.tensor(cuts, dtype=torch.int64, device=dev)


def distribute_codes(local_codes: torch.Tensor, splitters: torch.Tensor, group=None) -> torch.Tensor:
    """This rank's owned voxels: every rank's codes sent to their owners (one all-to-all), merged and uniqued."""
    world, _ = _world(group)
    owner = _owner_of(local_codes, splitters)
    order = torch.argsort(owner, stable=True)
    counts = torch.bincount(owner, minlength=world)
    recv, _ = _alltoallv(local_codes[order], counts.tolist(), group)
    return torch.unique(recv)


NEIGHBOUR_OFFSETS = [(dx, dy, dz) for dx in (-1, 0, 1) for dy in (-1, 0, 1) for dz in (-1, 0, 1)
                     if (dx, dy, dz) != (0, 0, 0)]


class LevelShard:
    """One level of a Morton-sharded voxel set, built from this rank's owned codes alone.

    owned_codes: this rank's voxels, sorted unique Morton codes inside [splitters[rank], splitters[rank + 1]).
    nmap_fn(coords [M, 4] int32, extents) -> tap-major [27, M] int32 neighbour map of a voxel set (the library's hash
    builder on GPUs, the oracle in the CPU tests).  The plan (`self.plan`, a ShardPlan) has the local row space
    [owned rows | halo rows], the owned rows' neighbour map in it, and the halo exchange lists; `offset` is the global
    index of the first owned voxel (global indices follow Morton order over all ranks)."""

    def __init__(self, owned_codes: torch.Tensor, splitters: torch.Tensor, nmap_fn, group=None):
        import torch.distributed as dist
        world, rank = _world(group)
        dev = owned_codes.device
        self.codes = owned_codes
        self.splitters = splitters
        n_own = int(owned_codes.numel())
        counts = torch.tensor([n_own], dtype=torch.int64, device=dev)
        if world > 1:
            parts = [torch.empty_like(counts) for _ in range(world)]
            dist.all_gather(parts, counts, group=group)
            allc = torch.cat(parts)
        else:
            allc = counts
        self.counts = [int(c) for c in allc.tolist()]
        self.offset = sum(self.counts[:rank])
        lo, hi = int(splitters[rank]), int(splitters[rank + 1])
        # neighbour candidates outside this rank's code range, each once, asked of their owners
        x, y, z = demorton3(owned_codes)
        limit = (1 << MORTON_BITS) - 1
        cand = []
        for dx, dy, dz in NEIGHBOUR_OFFSETS:
            nx, ny, nz = x + dx, y + dy, z + dz
            ok = (nx >= 0) & (ny >= 0) & (nz >= 0) & (nx <= limit) & (ny <= limit) & (nz <= limit)
            c = morton3(nx[ok], ny[ok], nz[ok])
            cand.append(c[(c < lo) | (c >= hi)])
        ask = torch.unique(torch.cat(cand)) if cand else owned_codes[:0]
        owner = _owner_of(ask, splitters)
        ask_counts = torch.bincount(owner, minlength=world).tolist()
        asked, asked_counts = _alltoallv(ask, ask_counts, group)          # codes other ranks ask this rank about
        pos = torch.searchsorted(owned_codes, asked)
        found = (pos < n_own) & (owned_codes[pos.clamp(max=max(n_own - 1, 0))] == asked) if n_own else \
            torch.zeros_like(asked, dtype=torch.bool)
        reply = torch.where(found, pos, torch.full_like(pos, -1))
        back, _ = _alltoallv(reply, asked_counts, group)                  # for each of this rank's questions
        exists = back >= 0
        halo_codes = ask[exists]                                          # sorted by code = by owner, global order
        self.halo_codes = halo_codes
        # send lists: the owned rows each peer found, in the peer's (sorted) halo order
        send_idx, send_splits, off = [], [], 0
        for c in asked_counts:
            r = reply[off:off + c]
            r = r[r >= 0]
            send_idx.append(r)
            send_splits.append(int(r.numel()))
            off += c
        recv_splits = torch.bincount(owner[exists], minlength=world).tolist()
        # the owned rows' neighbour map over owned + halo voxels, in the local row space
        local_codes = torch.cat([owned_codes, halo_codes])
        if local_codes.numel():
            nm = nmap_fn(coords_of_codes(local_codes), [1, 1 << MORTON_BITS, 1 << MORTON_BITS, 1 << MORTON_BITS])
        else:
            nm = torch.empty((27, 0), dtype=torch.int32, device=dev)
        self.plan = ShardPlan.from_parts(nm[:, :n_own].contiguous(), n_own, int(halo_codes.numel()), recv_splits,
                                         torch.cat(send_idx).to(torch.int64) if send_idx else reply[:0],
                                         send_splits, rank, world, group)


class PoolPlan:
    """The mean pool of level k's owned rows into the parents level k + 1 owns (code >> 3; flex_gemm's mean pool,
    children summed in code order), planned once per structure.  A parent's eight possible children are one Morton
    range: when that range lies inside this rank's level-k range, all of the parent's children are here, and the
    parent is pooled here (segment `pool_seg_*`) even when another rank owns it -- only the pooled row travels.  Only
    a parent whose children straddle a range boundary has raw children sent to its owner, which pools them together
    with its own in code order (`seg_*` over [owned rows | received rows]).  Pooled and raw rows go in ONE all-to-all,
    grouped by destination.  The sums and their order are those of a single-device pool, so results are identical."""

    def __init__(self, level: "LevelShard", next_level: "LevelShard", group=None):
        world, rank = _world(group)
        self.group, self.world = group, world
        codes = level.codes
        dev = codes.device
        self.n_own = n_own = int(codes.numel())
        parents = codes >> 3
        powner = _owner_of(parents, next_level.splitters)
        lo, hi = int(level.splitters[rank]), int(level.splitters[rank + 1])
        pu, inv, cnt = torch.unique_consecutive(parents, return_inverse=True, return_counts=True)
        first = torch.cumsum(cnt, 0) - cnt
        gown = powner[first] if n_own else powner[:0]
        complete = ((pu << 3) >= lo) & ((pu << 3) + 7 < hi)
        # parents pooled here for another rank, grouped by destination (code order within)
        pg = torch.nonzero((gown != rank) & complete).flatten()
        pg = pg[torch.argsort(gown[pg], stable=True)]
        self.n_pool_send = int(pg.numel())
        self.pool_seg_off = torch.zeros(self.n_pool_send + 1, dtype=torch.int32, device=dev)
        self.pool_seg_off[1:] = torch.cumsum(cnt[pg], 0).to(torch.int32)
        # a group's children are consecutive owned rows: first[g] + 0 .. cnt[g] - 1
        starts = torch.repeat_interleave(self.pool_seg_off[:-1].long(), cnt[pg])
        base = torch.repeat_interleave(first[pg], cnt[pg])
        self.pool_seg_idx = (base + torch.arange(int(starts.numel()), device=dev) - starts).to(torch.int32)
        pool_send_counts = torch.bincount(gown[pg], minlength=world)
        # raw children of straddling parents owned elsewhere, grouped by destination (code order within)
        raw_child = ((gown != rank) & ~complete)[inv] if n_own else torch.zeros(0, dtype=torch.bool, device=dev)
        rc = torch.nonzero(raw_child).flatten()
        rc = rc[torch.argsort(powner[rc], stable=True)]
        self.raw_send_idx = rc
        raw_send_counts = torch.bincount(powner[rc], minlength=world)
        # metadata: which parents arrive pooled, which children arrive raw
        got_p, pool_recv = _alltoallv(pu[pg], pool_send_counts.tolist(), group)
        got_c, raw_recv = _alltoallv(codes[rc], raw_send_counts.tolist(), group)
        # one all-to-all of rows: to each destination its pooled rows, then its raw children
        ps, rs_ = pool_send_counts.tolist(), raw_send_counts.tolist()
        perm, po, ro = [], 0, 0
        for d in range(world):
            perm.append(torch.arange(po, po + ps[d], device=dev))
            perm.append(self.n_pool_send + torch.arange(ro, ro + rs_[d], device=dev))
            po += ps[d]
            ro += rs_[d]
        self.send_perm = torch.cat(perm) if perm else torch.zeros(0, dtype=torch.int64, device=dev)
        self.send_splits = [a + b for a, b in zip(ps, rs_)]
        self.recv_splits = [a + b for a, b in zip(pool_recv, raw_recv)]
        self.n_recv = sum(self.recv_splits)
        # positions (in the received rows) of the pooled rows and of the raw children
        pool_pos, raw_pos, off = [], [], 0
        for a, b in zip(pool_recv, raw_recv):
            pool_pos.append(torch.arange(off, off + a, device=dev))
            raw_pos.append(torch.arange(off + a, off + a + b, device=dev))
            off += a + b
        pool_pos = torch.cat(pool_pos) if pool_pos else torch.zeros(0, dtype=torch.int64, device=dev)
        raw_pos = torch.cat(raw_pos) if raw_pos else torch.zeros(0, dtype=torch.int64, device=dev)
        self.recv_pool_pos = pool_pos
        # segments of the parents pooled here for this rank: own children (complete or not) + raw children received
        keep_idx = torch.nonzero(powner == rank).flatten()
        cand_idx = torch.cat([keep_idx, n_own + raw_pos])
        cand_codes = torch.cat([codes[keep_idx], got_c])
        srt = torch.argsort(cand_codes, stable=True)                     # children in code order
        self.seg_idx = cand_idx[srt].to(torch.int32).contiguous()
        seg_p, seg_cnt = torch.unique_consecutive(cand_codes[srt] >> 3, return_counts=True)
        self.n_seg = int(seg_p.numel())
        self.seg_off = torch.zeros(self.n_seg + 1, dtype=torch.int32, device=dev)
        self.seg_off[1:] = torch.cumsum(seg_cnt, 0).to(torch.int32)
        self.n_parents = int(next_level.codes.numel())
        # where each pooled row lands among the owned parents
        self.seg_out = torch.searchsorted(next_level.codes, seg_p)
        self.recv_out = torch.searchsorted(next_level.codes, got_p)
        allp = torch.sort(torch.cat([seg_p, got_p])).values
        if not torch.equal(allp, next_level.codes):
            raise RuntimeError("pooled parents differ from the next level's owned voxels")
        self.identity = self.n_seg == self.n_parents and not got_p.numel()

    def buffer(self, C: int, device) -> torch.Tensor:
        """[n_own + n_recv, C] fp32: the owned rows, then the rows other ranks send."""
        return torch.empty((self.n_own + self.n_recv, C), dtype=torch.float32, device=device)

    def apply(self, buf: torch.Tensor) -> torch.Tensor:
        """Pool `buf` (owned rows written by the caller) into the owned parents' means [n_parents, C] fp32."""
        import torch.distributed as dist
        if self.world > 1:                  # every rank enters the all-to-all, also with nothing to move
            own = buf[:self.n_own]
            pooled = _pool(own, self.pool_seg_idx, self.pool_seg_off, self.n_pool_send)
            send = torch.cat([pooled, own.index_select(0, self.raw_send_idx)]).index_select(0, self.send_perm)
            dist.all_to_all_single(buf[self.n_own:], send, self.recv_splits, self.send_splits, group=self.group)
        rows = _pool(buf, self.seg_idx, self.seg_off, self.n_seg)
        if self.identity:
            return rows
        out = torch.empty((self.n_parents, buf.shape[1]), dtype=buf.dtype, device=buf.device)
        out.index_copy_(0, self.seg_out, rows)
        if self.recv_pool_pos.numel():
            out.index_copy_(0, self.recv_out, buf[self.n_own:].index_select(0, self.recv_pool_pos))
        return out


def _pool(buf: torch.Tensor, seg_idx: torch.Tensor, seg_off: torch.Tensor, n: int) -> torch.Tensor:
    """Mean of every segment's rows of `buf`, summed in segment order (the pooling kernel on the GPU)."""
    from . import ops
    if n == 0:
        return buf[:0]
    if buf.is_cuda:
        return ops.pool_mean(buf, seg_idx, seg_off, n)
    rows = buf[seg_idx.long()]
    return torch.stack([_mean_in_order(rows[int(a):int(b)]) for a, b in zip(seg_off[:-1], seg_off[1:])])


def _mean_in_order(rows: torch.Tensor) -> torch.Tensor:
    """fl(sum in row order / n) in fp32 (the pooling kernels' arithmetic), on the CPU."""
    acc = torch.zeros(rows.shape[1], dtype=torch.float32)
    for r in rows:
        acc = acc + r
    return acc / torch.tensor(float(rows.shape[0]), dtype=torch.float32)


# Relative cost of one voxel at each level of the sharded encoder (two convs, the pool into it and its link; measured
# per voxel on one B200 with Model A's widths), used to balance the aligned ranges.
LEVEL_COST = (0.68, 1.05, 2.09, 5.8, 7.1)


def _level0_weights(codes: torch.Tensor, levels: int, cost=LEVEL_COST) -> torch.Tensor:
    """Per level-0 voxel (sorted unique codes): its own cost plus, at every coarser level, its ancestor's cost shared
    among the ancestor's level-0 descendants on this rank."""
    w = torch.full(codes.shape, float(cost[0]), dtype=torch.float64, device=codes.device)
    for k in range(1, levels):
        _, inv, cnt = torch.unique_consecutive(codes >> (3 * k), return_inverse=True, return_counts=True)
        w += float(cost[min(k, len(cost) - 1)]) / cnt[inv].to(torch.float64)
    return w


def build_levels(local_codes: torch.Tensor, levels: int, nmap_fn, group=None, aligned: bool = False) -> list:
    """Every level of a fused scene sharded by Morton ranges, from this rank's own back-projected codes.  Level 0:
    codes to the owners of sample-balanced ranges, then once more to final ranges; each coarser level: the parents
    (code >> 3) of the level below, sent to their owners.
    By default every level's ranges are balanced by that level's own voxel count; a parent whose children sit on
    another rank is pooled there and only its pooled row moves (PoolPlan).  aligned: the coarser levels' ranges are
    the level-0 boundaries' parent codes (boundary >> 3 per level), so a parent's children all sit on its rank except
    at the one parent straddling a boundary and the pool moves almost nothing, with the level-0 ranges cut to balance
    the whole encoder's work (LEVEL_COST per voxel and level) -- each level then carries its own imbalance, which
    measured slightly slower at 2 GPUs (11.19 vs 11.01 ms per step).  Returns [LevelShard] per level."""
    owned = distribute_codes(local_codes, morton_splitters(local_codes, group), group)
    weights = _level0_weights(owned, levels) if aligned else None
    splitters = morton_splitters(owned, group, weights=weights)
    owned = distribute_codes(owned, splitters, group)
    lv = [LevelShard(owned, splitters, nmap_fn, group)]
    s0 = splitters
    for k in range(1, levels):
        cand = torch.unique(lv[-1].codes >> 3)
        if aligned:
            splitters = s0.clone()
            splitters[1:-1] = s0[1:-1] >> (3 * k)
        else:
            splitters = morton_splitters(cand, group)
        lv.append(LevelShard(distribute_codes(cand, splitters, group), splitters, nmap_fn, group))
    return lv


def encoder_layers(widths, convs_per_level: int, seed: int, device):
    """Seeded int8 layers of a sharded U-Net encoder with the given level widths: per level `convs_per_level`
    submanifold convs (weights [27, C, C]) and, between levels, a pooling transition's int8 linear ([C', C])."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    convs, links = [], []
    for k, C in enumerate(widths):
        lv = []
        for _ in range(convs_per_level):
            w = torch.randint(-127, 128, (27, C, C), generator=g, dtype=torch.int8)
            ws = torch.rand(C, generator=g) * (4e-4 * 32 / C) + 1e-5
            b = torch.randn(C, generator=g) * 0.1
            lv.append((w.to(device), ws.to(device), b.to(device), 0.05, 0.04))
        convs.append(lv)
        if k + 1 < len(widths):
            Cn = widths[k + 1]
            w = torch.randint(-127, 128, (Cn, C), generator=g, dtype=torch.int8)
            ws = torch.rand(Cn, generator=g) * (4e-3 * 32 / C) + 1e-4
            b = torch.randn(Cn, generator=g) * 0.1
            links.append((w.to(device), ws.to(device), b.to(device), 0.02, 0.04))
    return convs, links


_SCALARS = {}


def _device_scalar(v: float, device) -> torch.Tensor:
    """A 0-dim fp32 tensor of v on `device`, made once (a step captured in a CUDA graph may not copy from the host)."""
    key = (float(v), str(device))
    t = _SCALARS.get(key)
    if t is None:
        t = _SCALARS[key] = torch.tensor(float(v), dtype=torch.float32, device=device)
    return t


def encoder_forward(levels: list, q0: torch.Tensor, convs, links, conv, link, group=None, out_scale: float = 0.04,
                    pools=None, overlap: bool = False):
    """The sharded encoder pass: at every level its convs, each after a halo exchange of the int8 input rows, then
    (between levels) the mean pool into parents (rows dequantised with the last conv's output scale, children moved
    to their parent's owner and summed in code order, PoolPlan) and the transition's int8 linear.  conv(q_local,
    nmap, mask, layer) and link(pooled fp32, layer) give the next int8 rows.  `pools`: the PoolPlans of the
    transitions (built here when not given).  overlap: each exchange runs beside the interior rows' conv
    (ShardPlan.conv; measured slower on B200 at 2 and 4 GPUs, where the halo is a few percent of the rows, so off by
    default).  Returns the int8 rows of every level's owned voxels after its convs."""
    if pools is None:
        pools = [PoolPlan(levels[k], levels[k + 1], group) for k in range(len(levels) - 1)]
    scale = _device_scalar(out_scale, q0.device)
    outs = []
    q = q0
    for k, lvl in enumerate(levels):
        plan = lvl.plan
        buf = plan.local_buffer(q.shape[1], q.dtype)
        buf[:plan.n_own] = q
        for layer in convs[k]:
            plan.conv(buf, layer, conv, overlap)
        q = buf[:plan.n_own]
        outs.append(q)
        if k + 1 < len(levels):
            pb = pools[k].buffer(q.shape[1], q.device)
            torch.mul(q, scale, out=pb[:plan.n_own])                  # dequantise into the pool buffer
            q = link(pools[k].apply(pb), links[k])
    return outs


def gpu_link(pooled: torch.Tensor, layer):
    """A pooling transition on the device: quantise the pooled means with the linear's input scale, then the dense
    int8 layer with the SiLU + requantise epilogue."""
    from . import ops
    w, ws, b, sa, s_out = layer
    if pooled.shape[0] == 0:
        return torch.empty((0, w.shape[0]), dtype=torch.int8, device=pooled.device)
    qp = ops.quantize(pooled.contiguous(), sa)
    return ops.dense_i8(qp, w, ws, b, sa, ops.EPI_SILU_Q8, s_out)
