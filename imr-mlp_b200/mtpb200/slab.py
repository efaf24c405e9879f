"""Slab decomposition of one periodic box with a ghost-atom halo exchange.

The box is cut into slabs along its first lattice direction (by the
fractional coordinate of each atom), one slab per rank.  A rank holds only
its own atoms plus ghost copies of the atoms of its two neighbouring slabs
that lie within `halo` = r_c + skin of its slab faces, exactly as a LAMMPS
domain decomposition with `newton_pair on` does for the reference's pair
style (LAMMPS/USER-MLIP/pair_MLIP_gpu_direct.cpp:457: full list, ghost
forces returned by reverse communication).

The rank's atoms form one local periodic structure for the library: the
cell's first lattice vector is stretched to cover the slab, both halo layers
and an empty gap of one more halo thickness, so that no pair forms across the
stretched direction; the other two directions keep the box's periodicity.
Owned atoms come first and the library evaluates only them as centres
(mtpb_set_center_count), with neighbours drawn from owned and ghost atoms.
One EFS step is then

  1. forward exchange: the current positions of the atoms in the halo layers
     go to the neighbouring ranks (one message per neighbour);
  2. EFS of the owned centres: forces for owned and ghost atoms (partial sums);
  3. reverse exchange: ghost forces go back to their owners and are added;
  4. all-reduce of the 10 totals (energy and virial).

At a neighbour-list rebuild, atoms that left the slab move to the
neighbouring rank (positions, types, ids and their per-atom payload), and the
halo send lists are rebuilt from the new positions.  Per-step traffic is the
halo (two layers of thickness r_c + skin), and per-rank memory is the slab
plus its halo: both shrink as 1/N.

The exchanges are written as phases: `pack_*` returns one tensor per
neighbouring rank, `unpack_*` consumes the tensors received from them, and
`p2p_exchange` moves them with grouped torch.distributed P2P operations
(ncclSend/ncclRecv on GPUs, gloo on the CPU).  `LocalRanks` runs every rank
of a decomposition inside one process by handing the packed tensors over
directly (tests).  No kernel reads another GPU's memory: every transfer lands
in a local buffer.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np


def _torch():
    import torch
    return torch


def interplanar_spacing(cell: np.ndarray) -> float:
    """Distance between the lattice planes spanned by the 2nd and 3rd cell
    vectors (the thickness of the box along its first direction)."""
    cell = np.asarray(cell, dtype=np.float64).reshape(3, 3)
    return abs(float(np.linalg.det(cell))) / float(np.linalg.norm(np.cross(cell[1], cell[2])))


class SlabDomain:
    """One rank's slab of a periodic box and its ghost layers.

    State (torch tensors on `device`): owned positions `pos` [n_own, 3] in the
    box's Cartesian frame (continuous between rebuilds), `types` [n_own],
    global atom `ids` [n_own], and an optional per-atom float64 `payload`
    [n_own, P] that migrates with the atoms (a reference position, say).
    Ghost layers: `n_ghost_lo` atoms from the lower neighbour then
    `n_ghost_hi` from the upper one, with their types and ids.
    """

    def __init__(self, cell, nranks: int, rank: int, halo: float, device=None):
        torch = _torch()
        if nranks < 2:
            raise ValueError("a slab decomposition needs at least two ranks")
        self.cell = np.asarray(cell, dtype=np.float64).reshape(3, 3)
        self.inv = np.linalg.inv(self.cell)
        self.nranks, self.rank = nranks, rank
        self.device = device if device is not None else torch.device("cpu")
        self.spacing = interplanar_spacing(self.cell)
        self.h = float(halo) / self.spacing          # halo thickness, fractional
        self.width = 1.0 / nranks
        if self.h > self.width:
            raise ValueError(f"slabs of {self.width * self.spacing:.3f} A are thinner than the "
                             f"halo of {halo:.3f} A: use fewer ranks")
        self.lo, self.hi = rank * self.width, (rank + 1) * self.width
        self.lower, self.upper = (rank - 1) % nranks, (rank + 1) % nranks
        # a gap of one halo (plus a margin for atoms that drift between
        # rebuilds) keeps the stretched direction free of pairs
        self.extent = self.width + 2.0 * self.h + 1.05 * self.h
        self.local_cell = self.cell.copy()
        self.local_cell[0] *= self.extent
        self.origin = (self.lo - self.h) * self.cell[0]
        a = self.cell[0]
        # Cartesian shift of each ghost block in the box frame: the lower
        # neighbour of rank 0 and the upper neighbour of the last rank sit
        # across the periodic boundary
        self.shift_lo = -a if rank == 0 else np.zeros(3)
        self.shift_hi = a if rank == nranks - 1 else np.zeros(3)
        dt = torch.float64
        self._inv_t = torch.as_tensor(self.inv, dtype=dt, device=self.device)
        self._cell_t = torch.as_tensor(self.cell, dtype=dt, device=self.device)
        self._origin_t = torch.as_tensor(self.origin, dtype=dt, device=self.device)
        self.peers: List[int] = sorted({self.lower, self.upper})
        self.pos = self.types = self.ids = self.payload = None
        self.send_idx: Dict[int, object] = {}
        self.n_ghost_lo = self.n_ghost_hi = 0
        self.ghost_types = self.ghost_ids = None
        self._ghost_shift = None
        self.rebuilds = 0
        self.migrated = 0

    # ---- ownership -----------------------------------------------------
    def _frac_x(self, pos):
        return pos @ self._inv_t[:, 0]

    def assign(self, positions, types, ids=None, payload=None):
        """Keeps the atoms of this rank's slab out of a whole box (set-up)."""
        torch = _torch()
        pos = torch.as_tensor(np.asarray(positions), dtype=torch.float64, device=self.device)
        fx = self._frac_x(pos)
        fx = fx - torch.floor(fx)
        slab = torch.clamp((fx * self.nranks).long(), max=self.nranks - 1)
        keep = torch.nonzero(slab == self.rank).flatten()
        n = pos.shape[0]
        all_ids = (torch.arange(n, device=self.device) if ids is None
                   else torch.as_tensor(np.asarray(ids), dtype=torch.int64, device=self.device))
        self.pos = self._wrap_x(pos[keep])
        self.types = torch.as_tensor(np.asarray(types), dtype=torch.int32,
                                     device=self.device)[keep]
        self.ids = all_ids[keep]
        self.payload = None if payload is None else torch.as_tensor(
            np.asarray(payload), dtype=torch.float64, device=self.device)[keep]

    def _wrap_x(self, pos):
        """Wraps positions into [0, 1) along the first lattice direction."""
        torch = _torch()
        fx = self._frac_x(pos)
        return pos - torch.floor(fx).unsqueeze(1) * self._cell_t[0]

    @property
    def n_own(self) -> int:
        return int(self.pos.shape[0])

    @property
    def n_ghost(self) -> int:
        return self.n_ghost_lo + self.n_ghost_hi

    # ---- migration (rebuild, phase 1) ------------------------------------
    def pack_migration(self):
        """Atoms that left the slab, grouped per destination neighbour:
        returns ({peer: count tensor [1]}, {peer: float64 [m, 5 + P]} rows of
        x, y, z, type, id, payload...).  The atoms are removed from this rank."""
        torch = _torch()
        self.pos = self._wrap_x(self.pos)
        fx = self._frac_x(self.pos)
        slab = torch.clamp((fx * self.nranks).long(), max=self.nranks - 1)
        # destination code: 0 stays, 1 goes to the lower neighbour, 2 to the
        # upper one (one neighbour at two ranks), 3 is further away; one
        # host read of the counts, the index lists by a stable sort
        code = torch.full_like(slab, 3)
        code = torch.where(slab == self.upper, 2 if self.lower != self.upper else 1, code)
        code = torch.where(slab == self.lower, 1, code)
        code = torch.where(slab == self.rank, 0, code)
        n_stay, n_lo, n_hi, n_far = torch.bincount(code, minlength=4).tolist()
        if n_far:
            raise RuntimeError("an atom moved further than one slab between rebuilds")
        order = torch.argsort(code, stable=True)
        keep = order[:n_stay]
        moving = {self.lower: order[n_stay:n_stay + n_lo]}
        if self.upper != self.lower:
            moving[self.upper] = order[n_stay + n_lo:n_stay + n_lo + n_hi]
        counts, rows = {}, {}
        for p in self.peers:
            idx = moving[p]
            cols = [self.pos[idx], self.types[idx].double().unsqueeze(1),
                    self.ids[idx].double().unsqueeze(1)]
            if self.payload is not None:
                cols.append(self.payload[idx])
            rows[p] = torch.cat(cols, dim=1)
            counts[p] = torch.tensor([idx.numel()], dtype=torch.int64, device=self.device)
        self.migrated = n_lo + n_hi
        self.pos, self.types, self.ids = self.pos[keep], self.types[keep], self.ids[keep]
        if self.payload is not None:
            self.payload = self.payload[keep]
        return counts, rows

    def row_width(self) -> int:
        return 5 + (0 if self.payload is None else int(self.payload.shape[1]))

    def unpack_migration(self, rows: Dict[int, object]):
        """Appends the atoms received from the neighbours."""
        torch = _torch()
        parts = [rows[p] for p in self.peers if rows.get(p) is not None and rows[p].shape[0]]
        if not parts:
            return
        r = torch.cat(parts)
        self.pos = torch.cat([self.pos, self._wrap_x(r[:, 0:3].contiguous())])
        self.types = torch.cat([self.types, r[:, 3].round().to(torch.int32)])
        self.ids = torch.cat([self.ids, r[:, 4].round().to(torch.int64)])
        if self.payload is not None:
            self.payload = torch.cat([self.payload, r[:, 5:].contiguous()])

    # ---- halo lists (rebuild, phase 2) -------------------------------------
    def pack_halo(self):
        """Builds the send lists from the current positions and returns
        ({peer: count tensor [2]}, {peer: int64 [m, 2] rows of type, id}).
        Message to peer p: its lower-ghost segment (my atoms within the halo
        of my upper face, if p is my upper neighbour) then its upper-ghost
        segment (my atoms within the halo of my lower face, if p is my lower
        neighbour); counts hold both segment sizes."""
        torch = _torch()
        fx = self._frac_x(self.pos)
        m_lo = fx < self.lo + self.h
        m_hi = fx >= self.hi - self.h
        c_lo, c_hi = torch.stack([m_lo.sum(), m_hi.sum()]).tolist()   # one host read
        near_lo = torch.argsort((~m_lo).to(torch.int8), stable=True)[:c_lo]
        near_hi = torch.argsort((~m_hi).to(torch.int8), stable=True)[:c_hi]
        empty = torch.zeros(0, dtype=torch.int64, device=self.device)
        counts, rows = {}, {}
        self.send_idx = {}
        for p in self.peers:
            seg_a = near_hi if p == self.upper else empty   # p's lower ghosts
            seg_b = near_lo if p == self.lower else empty   # p's upper ghosts
            idx = torch.cat([seg_a, seg_b])
            self.send_idx[p] = idx
            counts[p] = torch.tensor([seg_a.numel(), seg_b.numel()], dtype=torch.int64,
                                     device=self.device)
            rows[p] = torch.stack([self.types[idx].long(), self.ids[idx]], dim=1)
        return counts, rows

    def unpack_halo(self, counts: Dict[int, object], rows: Dict[int, object]):
        """Lays out the ghosts: [lower block | upper block]."""
        torch = _torch()
        lo_parts, hi_parts = [], []
        self._recv_split = {}
        for q in self.peers:
            c = counts[q] if isinstance(counts[q], list) else [int(v) for v in counts[q].tolist()]
            r = rows[q]
            # q's message: [my lower ghosts (q is my lower), my upper ghosts (q is my upper)]
            self._recv_split[q] = c
            if q == self.lower:
                lo_parts.append(r[:c[0]])
            if q == self.upper:
                hi_parts.append(r[c[0]:c[0] + c[1]])
        cat = lambda ps: torch.cat(ps) if ps else torch.zeros((0, 2), dtype=torch.int64,   # noqa: E731
                                                              device=self.device)
        lo, hi = cat(lo_parts), cat(hi_parts)
        self.n_ghost_lo, self.n_ghost_hi = int(lo.shape[0]), int(hi.shape[0])
        g = torch.cat([lo, hi])
        self.ghost_types = g[:, 0].to(torch.int32)
        self.ghost_ids = g[:, 1]
        sl = torch.as_tensor(self.shift_lo, dtype=torch.float64, device=self.device)
        sh = torch.as_tensor(self.shift_hi, dtype=torch.float64, device=self.device)
        self._ghost_shift = torch.cat([sl.expand(self.n_ghost_lo, 3),
                                       sh.expand(self.n_ghost_hi, 3)]) - self._origin_t
        # per-step buffers: the local positions (the ghosts are received in
        # place), one send buffer per neighbour, the returned ghost forces
        n = self.n_own
        self._local = torch.empty((n + self.n_ghost, 3), dtype=torch.float64, device=self.device)
        self._send = {p: torch.empty((int(idx.numel()), 3), dtype=torch.float64,
                                     device=self.device) for p, idx in self.send_idx.items()}
        self._frecv = {p: torch.empty((int(idx.numel()), 3), dtype=torch.float64,
                                      device=self.device) for p, idx in self.send_idx.items()}
        self.rebuilds += 1

    def recv_halo_counts(self):
        """Shapes of the halo-count messages expected from each neighbour."""
        return {q: ((2,), "int64") for q in self.peers}

    # ---- per step: forward positions, reverse forces ----------------------
    def send_counts(self) -> Dict[int, int]:
        return {p: int(idx.numel()) for p, idx in self.send_idx.items()}

    def recv_counts(self) -> Dict[int, int]:
        return {q: sum(c) if (q == self.lower and q == self.upper) else
                (c[0] if q == self.lower else c[1]) for q, c in self._recv_split.items()}

    def _ghost_rows(self, q):
        """Row range of the local arrays that peer q's message covers: its
        lower-ghost segment and / or its upper-ghost segment, which are
        adjacent (the lower block, the upper block, or both at two ranks)."""
        n, lo, hi = self.n_own, self.n_ghost_lo, self.n_ghost_hi
        a = n if q == self.lower else n + lo
        b = n + lo + hi if q == self.upper else n + lo
        return a, b

    def pack_positions(self):
        """{peer: float64 [m, 3]} current positions of the halo atoms (into
        the send buffers; gathered in the order of the send lists)."""
        torch = _torch()
        out = {}
        for p, idx in self.send_idx.items():
            torch.index_select(self.pos, 0, idx, out=self._send[p])
            out[p] = self._send[p]
        return out

    def recv_views(self):
        """{peer: the rows of the local positions its message lands in}."""
        return {q: self._local[slice(*self._ghost_rows(q))] for q in self.peers}

    def finish_positions(self):
        """Local positions [owned | lower ghosts | upper ghosts] in the frame
        of the stretched local cell, once the ghost rows hold the received
        box-frame positions."""
        torch = _torch()
        n = self.n_own
        self._local[n:] += self._ghost_shift
        torch.sub(self.pos, self._origin_t, out=self._local[:n])
        return self._local

    def unpack_positions(self, msgs):
        for q, view in self.recv_views().items():
            view.copy_(msgs[q])
        return self.finish_positions()

    def local_types(self):
        return _torch().cat([self.types, self.ghost_types])

    def pack_forces(self, forces):
        """{peer: float64 [m, 3]} ghost rows of the local forces, in the
        order the peer sent those atoms (views, no copy)."""
        return {q: forces[slice(*self._ghost_rows(q))] for q in self.peers}

    def force_recv_buffers(self):
        return self._frecv

    def unpack_forces(self, forces, msgs):
        """Owned forces: own rows plus the ghost forces returned by the
        neighbours (newton-on reverse communication), added in place into
        the owned rows of `forces`; returns that view."""
        f = forces[:self.n_own]
        for p, idx in self.send_idx.items():
            if idx.numel():
                f.index_add_(0, idx, msgs[p])
        return f


# ---- transports ---------------------------------------------------------
def p2p_exchange(dist, sends: Dict[int, object], recv_shapes: Dict[int, tuple], dtype, device,
                 group=None):
    """Grouped send/receive of one tensor per peer (ncclSend/ncclRecv inside
    one group on NCCL).  Empty messages are skipped on both sides (their sizes
    are known to both)."""
    torch = _torch()
    recvs = {q: torch.empty(shape, dtype=dtype, device=device) for q, shape in
             recv_shapes.items()}
    return p2p_exchange_into(dist, sends, recvs, group)


def p2p_exchange_into(dist, sends: Dict[int, object], recvs: Dict[int, object], group=None):
    """p2p_exchange into preallocated (contiguous) receive tensors."""
    ops = []
    for p, t in sends.items():
        if t.numel():
            ops.append(dist.P2POp(dist.isend, t.contiguous(), p, group))
    for q, t in recvs.items():
        if t.numel():
            ops.append(dist.P2POp(dist.irecv, t, q, group))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return recvs


class DistributedSlab:
    """Drives one SlabDomain over a torch.distributed process group."""

    def __init__(self, domain: SlabDomain, dist, group=None):
        self.d = domain
        self.dist = dist
        self.group = group

    def rebuild(self):
        torch = _torch()
        d = self.d
        counts, rows = d.pack_migration()
        rc = p2p_exchange(self.dist, counts, {q: (1,) for q in d.peers}, torch.int64, d.device,
                          self.group)
        n_in = torch.cat([rc[q] for q in d.peers]).tolist()   # one host read
        w = d.row_width()
        recv = p2p_exchange(self.dist, rows, {q: (n, w) for q, n in zip(d.peers, n_in)},
                            torch.float64, d.device, self.group)
        d.unpack_migration(recv)
        counts, rows = d.pack_halo()
        hc = p2p_exchange(self.dist, counts, {q: (2,) for q in d.peers}, torch.int64, d.device,
                          self.group)
        flat = torch.cat([hc[q] for q in d.peers]).tolist()   # one host read
        hcl = {q: flat[2 * k:2 * k + 2] for k, q in enumerate(d.peers)}
        hr = p2p_exchange(self.dist, rows, {q: (sum(hcl[q]), 2) for q in d.peers},
                          torch.int64, d.device, self.group)
        d.unpack_halo(hcl, hr)

    def positions(self):
        d = self.d
        p2p_exchange_into(self.dist, d.pack_positions(), d.recv_views(), self.group)
        return d.finish_positions()

    def forces(self, local_forces):
        d = self.d
        msgs = p2p_exchange_into(self.dist, d.pack_forces(local_forces), d.force_recv_buffers(),
                                 self.group)
        return d.unpack_forces(local_forces, msgs)

    def totals(self, t):
        self.dist.all_reduce(t, group=self.group)
        return t


class LocalRanks:
    """Every rank of a decomposition in one process: the packed tensors are
    handed to their receivers directly."""

    def __init__(self, domains: List[SlabDomain]):
        self.ds = domains

    @staticmethod
    def _route(sends: List[Dict[int, object]]):
        return [{p: sends[p][r] for p in sends[r].keys()} for r in range(len(sends))]

    def rebuild(self):
        mig = [d.pack_migration()[1] for d in self.ds]
        for d, got in zip(self.ds, self._route(mig)):
            d.unpack_migration(got)
        halo = [d.pack_halo() for d in self.ds]
        counts = self._route([h[0] for h in halo])
        rows = self._route([h[1] for h in halo])
        for d, c, r in zip(self.ds, counts, rows):
            d.unpack_halo(c, r)

    def positions(self):
        msgs = self._route([d.pack_positions() for d in self.ds])
        return [d.unpack_positions(m) for d, m in zip(self.ds, msgs)]

    def forces(self, local_forces):
        msgs = self._route([d.pack_forces(f) for d, f in zip(self.ds, local_forces)])
        return [d.unpack_forces(f, m) for d, f, m in zip(self.ds, local_forces, msgs)]


def local_structure(domain: SlabDomain, positions) -> dict:
    """The rank's atoms as one periodic structure for the library (numpy)."""
    return dict(cell=domain.local_cell.copy(), pbc=np.ones(3, np.int32),
                positions=positions.detach().cpu().numpy() if hasattr(positions, "detach")
                else np.asarray(positions),
                types=domain.local_types().cpu().numpy().astype(np.int32))


def halo_bytes_per_step(domain: SlabDomain) -> Dict[str, int]:
    """Bytes this rank sends per EFS step: ghost positions out (forward),
    ghost forces out (reverse), plus the 10-double all-reduce."""
    fwd = 24 * sum(domain.send_counts().values())
    rev = 24 * domain.n_ghost
    return {"forward": fwd, "reverse": rev, "totals": 80}


class SlabEFS:
    """One rank's EFS step of a slab decomposition through the library: the
    step a domain-decomposed MD code runs every time step.  `rebuild()` (every
    few steps) migrates atoms and remakes the halo, and the next `compute`
    rebuilds the neighbour lists of the local structure; `compute()` exchanges
    ghost positions, evaluates the owned centres (device arrays, the
    library's context stream), returns ghost forces to their owners and
    all-reduces energy and virial.  Returns (owned forces [n_own, 3],
    totals [10] = energy, virial row-major)."""

    def __init__(self, gpu, transport: DistributedSlab):
        torch = _torch()
        self.gpu = gpu
        self.t = transport
        self.d = transport.d
        dev = self.d.device
        self.totals = torch.zeros(10, dtype=torch.float64, device=dev)
        self._pbc = torch.ones((1, 3), dtype=torch.int32, device=dev)
        self._cell = torch.as_tensor(self.d.local_cell.reshape(1, 9), dtype=torch.float64,
                                     device=dev)
        self._built = False

    def rebuild(self):
        torch = _torch()
        d = self.d
        self.t.rebuild()
        n_local = d.n_own + d.n_ghost
        self.gpu.set_center_count(d.n_own)
        dev = d.device
        self._offs = torch.tensor([0, n_local], dtype=torch.int32, device=dev)
        self._types = d.local_types().contiguous()
        self._f = torch.zeros((n_local, 3), dtype=torch.float64, device=dev)
        self._built = False

    def compute(self):
        x = self.t.positions()
        # energy and virial land in the vector that is all-reduced
        self.gpu.efs_device(self._offs, self._cell, self._pbc, x, self._types,
                            self.totals[0:1], self._f, self.totals[1:].view(1, 9),
                            reuse_neighbors=self._built)
        self._built = True
        f_own = self.t.forces(self._f)
        self.t.totals(self.totals)
        return f_own, self.totals
