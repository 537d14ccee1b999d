"""Seeded generators of the benchmark tasks, written in the reference's normalized task text format
(include/mymyr/formalism/text_format.hpp in maichmueller/mymyr; sections O P SI FI G A). Types are static unary
predicates, as the reference's normalization compiles them. The random source is a self-contained splitmix64, so a
(generator, seed) pair always yields the same text; parity depends only on the emitted text.

    tower(7, seed=0)                   7-block tower stacking, full-space BrFS
    transport(2, 40, 2, seed=0)        two-room gripper transport for the batched env step (65,536 envs)
    sliding_tile(4, 4, 60, seed=0)     4x4 sliding tile, BrFS to depth 22 (the headline workload)
    random_domain(seed=0)              24 predicates, 16 schemas of 3-5 parameters, 200 typed objects (the lifted
                                       successor-generation stress test over bernoulli_rows batches)
    logistics(8, 4, 6, 2, 30, seed=0)  logistics for A* with h^max
"""

from __future__ import annotations

from dataclasses import dataclass, field

MASK = (1 << 64) - 1


class SplitMix:
    """splitmix64 (Steele, Lea, Flood 2014)."""

    def __init__(self, seed: int):
        self.s = seed & MASK

    def next(self) -> int:
        self.s = (self.s + 0x9E3779B97F4A7C15) & MASK
        z = self.s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK
        return z ^ (z >> 31)

    def below(self, n: int) -> int:
        return (self.next() * n) >> 64

    def shuffle(self, xs: list) -> list:
        xs = list(xs)
        for i in range(len(xs) - 1, 0, -1):
            j = self.below(i + 1)
            xs[i], xs[j] = xs[j], xs[i]
        return xs


@dataclass
class TaskText:
    """A task under construction; text() renders the format."""

    n: int = 0
    preds: list = field(default_factory=list)      # (kind, arity, name)
    static_init: list = field(default_factory=list)  # (pred, args)
    fluent_init: list = field(default_factory=list)
    goal: list = field(default_factory=list)       # (pred, positive, args)
    schemas: list = field(default_factory=list)    # (name, arity, pre, eff); literals (pred, positive, terms)

    def pred(self, kind: str, arity: int, name: str) -> int:
        self.preds.append((kind, arity, name))
        return len(self.preds) - 1

    def text(self) -> str:
        out = [f"O {self.n}", f"P {len(self.preds)}"]
        out += [f"{k} {a} {nm}" for k, a, nm in self.preds]
        for tag, atoms in (("SI", self.static_init), ("FI", self.fluent_init)):
            out.append(f"{tag} {len(atoms)}")
            out += [" ".join(str(x) for x in (p, *args)) for p, args in atoms]
        out.append(f"G {len(self.goal)}")
        out += [" ".join(str(x) for x in (p, int(pos), *args)) for p, pos, args in self.goal]
        out.append(f"A {len(self.schemas)}")
        for name, arity, pre, eff in self.schemas:
            out.append(f"{name} {arity}")
            out.append(f"L {len(pre)}")
            out += [" ".join(str(x) for x in (p, int(pos), *terms)) for p, pos, terms in pre]
            out += ["E 1", "0", "L 0", f"F {len(eff)}"]
            out += [" ".join(str(x) for x in (p, int(pos), *terms)) for p, pos, terms in eff]
        return "\n".join(out) + "\n"


def obj(o: int) -> int:
    """The term of object o."""
    return -(o + 1)


def _partition(rng: SplitMix, blocks: list[int]) -> list[list[int]]:
    order = rng.shuffle(blocks)
    stacks, cur = [], []
    for b in order:
        cur.append(b)
        if rng.below(3) == 0:
            stacks.append(cur)
            cur = []
    if cur:
        stacks.append(cur)
    return stacks


def tower(n_blocks: int = 7, seed: int = 0) -> str:
    """Blocks world with on/ontable/clear/handempty/holding and pick-up, put-down, stack, unstack (unit cost).
    Initial and goal configurations are random stack partitions (bottom first) drawn from the seed."""
    rng = SplitMix(seed)
    t = TaskText(n=n_blocks)
    on = t.pred("F", 2, "on")
    ontable = t.pred("F", 1, "ontable")
    clear = t.pred("F", 1, "clear")
    handempty = t.pred("F", 0, "handempty")
    holding = t.pred("F", 1, "holding")
    blocks = list(range(n_blocks))
    for stack in _partition(rng, blocks):
        t.fluent_init.append((ontable, (stack[0],)))
        for lo, hi in zip(stack, stack[1:]):
            t.fluent_init.append((on, (hi, lo)))
        t.fluent_init.append((clear, (stack[-1],)))
    t.fluent_init.append((handempty, ()))
    for stack in _partition(rng, blocks):
        t.goal.append((ontable, True, (stack[0],)))
        for lo, hi in zip(stack, stack[1:]):
            t.goal.append((on, True, (hi, lo)))
    t.schemas.append(("pick-up", 1, [(clear, 1, (0,)), (ontable, 1, (0,)), (handempty, 1, ())],
                      [(ontable, 0, (0,)), (clear, 0, (0,)), (handempty, 0, ()), (holding, 1, (0,))]))
    t.schemas.append(("put-down", 1, [(holding, 1, (0,))],
                      [(holding, 0, (0,)), (clear, 1, (0,)), (handempty, 1, ()), (ontable, 1, (0,))]))
    t.schemas.append(("stack", 2, [(holding, 1, (0,)), (clear, 1, (1,))],
                      [(holding, 0, (0,)), (clear, 0, (1,)), (clear, 1, (0,)), (handempty, 1, ()), (on, 1, (0, 1))]))
    t.schemas.append(("unstack", 2, [(on, 1, (0, 1)), (clear, 1, (0,)), (handempty, 1, ())],
                      [(holding, 1, (0,)), (clear, 1, (1,)), (clear, 0, (0,)), (handempty, 0, ()), (on, 0, (0, 1))]))
    return t.text()


def transport(n_rooms: int = 2, n_balls: int = 40, n_grippers: int = 2, seed: int = 0) -> str:
    """Gripper transport: a robot with grippers carries balls between rooms (at-robby, at, free, carry; move, pick,
    drop). Ball positions, their goal rooms and the robot's room are drawn from the seed."""
    rng = SplitMix(seed)
    t = TaskText(n=n_rooms + n_balls + n_grippers)
    room = t.pred("S", 1, "room")
    ball = t.pred("S", 1, "ball")
    gripper = t.pred("S", 1, "gripper")
    at_robby = t.pred("F", 1, "at-robby")
    at = t.pred("F", 2, "at")
    free = t.pred("F", 1, "free")
    carry = t.pred("F", 2, "carry")
    rooms = list(range(n_rooms))
    balls = list(range(n_rooms, n_rooms + n_balls))
    grippers = list(range(n_rooms + n_balls, n_rooms + n_balls + n_grippers))
    t.static_init += [(room, (r,)) for r in rooms] + [(ball, (b,)) for b in balls] + [(gripper, (g,)) for g in grippers]
    t.fluent_init.append((at_robby, (rooms[rng.below(n_rooms)],)))
    t.fluent_init += [(at, (b, rooms[rng.below(n_rooms)])) for b in balls]
    t.fluent_init += [(free, (g,)) for g in grippers]
    t.goal += [(at, True, (b, rooms[rng.below(n_rooms)])) for b in balls]
    t.schemas.append(("move", 2, [(room, 1, (0,)), (room, 1, (1,)), (at_robby, 1, (0,))],
                      [(at_robby, 1, (1,)), (at_robby, 0, (0,))]))
    t.schemas.append(("pick", 3, [(ball, 1, (0,)), (room, 1, (1,)), (gripper, 1, (2,)), (at, 1, (0, 1)),
                                  (at_robby, 1, (1,)), (free, 1, (2,))],
                      [(carry, 1, (0, 2)), (at, 0, (0, 1)), (free, 0, (2,))]))
    t.schemas.append(("drop", 3, [(ball, 1, (0,)), (room, 1, (1,)), (gripper, 1, (2,)), (carry, 1, (0, 2)),
                                  (at_robby, 1, (1,))],
                      [(at, 1, (0, 1)), (free, 1, (2,)), (carry, 0, (0, 2))]))
    return t.text()


def sliding_tile(rows: int = 4, cols: int = 4, scramble: int = 60, seed: int = 0) -> str:
    """The rows x cols sliding-tile puzzle in STRIPS: at(tile, pos), blank(pos), static adj(p, q); one schema
    move(t, from, to). The start is `scramble` seeded random blank moves from the solved layout (blank at p0, tile k at
    p_k); the goal is the solved layout."""
    rng = SplitMix(seed)
    ntiles, npos = rows * cols - 1, rows * cols
    t = TaskText(n=ntiles + npos)
    tile = t.pred("S", 1, "tile")
    pos = t.pred("S", 1, "pos")
    adj = t.pred("S", 2, "adj")
    at = t.pred("F", 2, "at")
    blank = t.pred("F", 1, "blank")
    P = lambda k: ntiles + k  # object of position k
    t.static_init += [(tile, (k,)) for k in range(ntiles)] + [(pos, (P(k),)) for k in range(npos)]

    def nbrs(k):
        r, c = divmod(k, cols)
        out = []
        for dr, dc in ((-1, 0), (1, 0), (0, -1), (0, 1)):
            rr, cc = r + dr, c + dc
            if 0 <= rr < rows and 0 <= cc < cols:
                out.append(rr * cols + cc)
        return out

    for k in range(npos):
        for q in nbrs(k):
            t.static_init.append((adj, (P(k), P(q))))
    layout = [None] + list(range(ntiles))  # layout[position] = tile (None: blank); tile k-1 solved at p_k
    b = 0
    for _ in range(scramble):
        ns = nbrs(b)
        q = ns[rng.below(len(ns))]
        layout[b], layout[q] = layout[q], None
        b = q
    for k in range(npos):
        if layout[k] is None:
            t.fluent_init.append((blank, (P(k),)))
        else:
            t.fluent_init.append((at, (layout[k], P(k))))
    t.goal += [(at, True, (k - 1, P(k))) for k in range(1, npos)]
    t.schemas.append(("move", 3, [(tile, 1, (0,)), (pos, 1, (1,)), (pos, 1, (2,)), (at, 1, (0, 1)), (blank, 1, (2,)),
                                  (adj, 1, (1, 2))],
                      [(at, 1, (0, 2)), (blank, 1, (1,)), (at, 0, (0, 1)), (blank, 0, (2,))]))
    return t.text()


def random_domain(seed: int = 0, n_types: int = 10, per_type: int = 20, n_unary: int = 6, n_binary: int = 14,
                  n_ternary: int = 4, n_schemas: int = 16, n_init: int = 4) -> str:
    """A synthetic typed STRIPS domain: n_types types of per_type objects (200 objects by default), 24 fluent
    predicates of arity 1-3 with random type signatures, and n_schemas schemas with 3-5 typed parameters, as many
    positive fluent preconditions as parameters plus 0-1 (3-6 in all, every parameter mentioned), and 2-4 add/delete
    effects. The precondition count scales with the parameters so that a state at 5% atom density keeps a bounded
    number of applicable actions. The initial state holds n_init atoms (4 by default: the stress test expands random
    states, not the initial one; a larger one gives a searchable space)."""
    rng = SplitMix(seed)
    n = n_types * per_type
    t = TaskText(n=n)
    types = [t.pred("S", 1, f"type{k}") for k in range(n_types)]
    t.static_init += [(types[o // per_type], (o,)) for o in range(n)]
    sigs = []  # (pred, [types])
    for arity, count in ((1, n_unary), (2, n_binary), (3, n_ternary)):
        for _ in range(count):
            sig = [rng.below(n_types) for _ in range(arity)]
            sigs.append((t.pred("F", arity, f"f{len(sigs)}"), sig))
    for s in range(n_schemas):
        for _attempt in range(1000):
            k = 3 + rng.below(3)
            ptypes = [rng.below(n_types) for _ in range(k)]
            by_type = {}
            for i, ty in enumerate(ptypes):
                by_type.setdefault(ty, []).append(i)
            usable = [(p, sig) for p, sig in sigs if all(ty in by_type for ty in sig)]
            if not usable:
                continue
            npre = min(6, k + rng.below(2))
            pre = []
            for _ in range(npre):
                p, sig = usable[rng.below(len(usable))]
                terms = tuple(by_type[ty][rng.below(len(by_type[ty]))] for ty in sig)
                pre.append((p, 1, terms))
            mentioned = {x for _, _, terms in pre for x in terms}
            if len(mentioned) < k or len(set(pre)) < len(pre):
                continue
            neff = 2 + rng.below(3)
            eff = []
            for _ in range(neff):
                if rng.below(2) == 0:  # delete one of the preconditions
                    p, _, terms = pre[rng.below(len(pre))]
                    eff.append((p, 0, terms))
                else:
                    p, sig = usable[rng.below(len(usable))]
                    terms = tuple(by_type[ty][rng.below(len(by_type[ty]))] for ty in sig)
                    eff.append((p, 1, terms))
            if len(set(eff)) < len(eff):
                continue
            typing = [(types[ptypes[i]], 1, (i,)) for i in range(k)]
            t.schemas.append((f"a{s}", k, typing + pre, eff))
            break
        else:
            raise RuntimeError("random_domain: could not draw a schema")
    # a small initial state and goal (the stress test expands random states, not the initial one)
    for p, sig in sigs[:4]:
        args = tuple(ty * per_type + rng.below(per_type) for ty in sig)
        t.fluent_init.append((p, args))
    seen = set(t.fluent_init)
    while len(t.fluent_init) < n_init:
        p, sig = sigs[rng.below(len(sigs))]
        atom = (p, tuple(ty * per_type + rng.below(per_type) for ty in sig))
        if atom not in seen:
            seen.add(atom)
            t.fluent_init.append(atom)
    p, sig = sigs[-1]
    t.goal.append((p, True, tuple(ty * per_type for ty in sig)))
    return t.text()


def logistics(n_cities: int = 8, locs_per_city: int = 4, n_trucks: int = 6, n_airplanes: int = 2,
              n_packages: int = 30, seed: int = 0) -> str:
    """Logistics: packages travel by truck between the locations of a city and by airplane between airports (the
    first location of every city); predicates at(object, location), in(package, vehicle), in-city(location, city)
    (static) plus type predicates and airport; schemas load, unload, drive, fly, unit cost. Trucks start in distinct
    cities (one per city while there are trucks); a package's origin and destination are drawn among the locations a
    truck or an airplane serves (the airport only, in a city without a truck), and differ."""
    rng = SplitMix(seed)
    C, L = n_cities, n_cities * locs_per_city
    cities = list(range(C))
    locs = list(range(C, C + L))
    trucks = list(range(C + L, C + L + n_trucks))
    planes = list(range(C + L + n_trucks, C + L + n_trucks + n_airplanes))
    pkgs = list(range(C + L + n_trucks + n_airplanes, C + L + n_trucks + n_airplanes + n_packages))
    t = TaskText(n=C + L + n_trucks + n_airplanes + n_packages)
    city = t.pred("S", 1, "city")
    location = t.pred("S", 1, "location")
    truck = t.pred("S", 1, "truck")
    airplane = t.pred("S", 1, "airplane")
    vehicle = t.pred("S", 1, "vehicle")
    package = t.pred("S", 1, "package")
    airport = t.pred("S", 1, "airport")
    in_city = t.pred("S", 2, "in-city")
    at = t.pred("F", 2, "at")
    inside = t.pred("F", 2, "in")
    city_of = {}
    for c in cities:
        t.static_init.append((city, (c,)))
        for k in range(locs_per_city):
            l = locs[c * locs_per_city + k]
            city_of[l] = c
            t.static_init.append((location, (l,)))
            t.static_init.append((in_city, (l, c)))
            if k == 0:
                t.static_init.append((airport, (l,)))
    for v in trucks:
        t.static_init += [(truck, (v,)), (vehicle, (v,))]
    for v in planes:
        t.static_init += [(airplane, (v,)), (vehicle, (v,))]
    for p in pkgs:
        t.static_init.append((package, (p,)))
    truck_cities = rng.shuffle(cities)[:n_trucks] if n_trucks <= C else [rng.below(C) for _ in trucks]
    for v, c in zip(trucks, truck_cities):
        t.fluent_init.append((at, (v, locs[c * locs_per_city + rng.below(locs_per_city)])))
    for v in planes:
        t.fluent_init.append((at, (v, locs[rng.below(C) * locs_per_city])))
    served = [l for l in locs if city_of[l] in set(truck_cities) or (l - C) % locs_per_city == 0]
    for p in pkgs:
        a = served[rng.below(len(served))]
        b = a
        while b == a:
            b = served[rng.below(len(served))]
        t.fluent_init.append((at, (p, a)))
        t.goal.append((at, True, (p, b)))
    t.schemas.append(("load", 3, [(package, 1, (0,)), (vehicle, 1, (1,)), (location, 1, (2,)), (at, 1, (1, 2)),
                                  (at, 1, (0, 2))],
                      [(at, 0, (0, 2)), (inside, 1, (0, 1))]))
    t.schemas.append(("unload", 3, [(package, 1, (0,)), (vehicle, 1, (1,)), (location, 1, (2,)), (at, 1, (1, 2)),
                                    (inside, 1, (0, 1))],
                      [(inside, 0, (0, 1)), (at, 1, (0, 2))]))
    t.schemas.append(("drive", 4, [(truck, 1, (0,)), (location, 1, (1,)), (location, 1, (2,)), (city, 1, (3,)),
                                   (at, 1, (0, 1)), (in_city, 1, (1, 3)), (in_city, 1, (2, 3))],
                      [(at, 0, (0, 1)), (at, 1, (0, 2))]))
    t.schemas.append(("fly", 3, [(airplane, 1, (0,)), (airport, 1, (1,)), (airport, 1, (2,)), (at, 1, (0, 1))],
                      [(at, 0, (0, 1)), (at, 1, (0, 2))]))
    return t.text()


def counters(n_counters: int = 3, modulus: int = 5, seed: int = 0) -> str:
    """Modular counters: each counter holds a value mod `modulus` (fluent val(counter, value)); static facts
    plus(a, b, c) for a + b = c (mod modulus) and le(a, b) for a <= b. Schemas: add(c1, c2, x, y, z) sets c1 to
    x + y through the ternary plus(x, y, z); double(c, x, z) through plus(x, x, z), a static literal with a repeated
    parameter; reset(c, x) back to value 0 under le(x, x). Initial values are drawn from the seed. Exercises the
    matchers' checks of static literals by key (arity 3 and repeated parameters), which the other workloads lack."""
    rng = SplitMix(seed)
    k, m = n_counters, modulus
    cs = list(range(k))
    vs = list(range(k, k + m))
    t = TaskText(n=k + m)
    counter = t.pred("S", 1, "counter")
    value = t.pred("S", 1, "value")
    plus = t.pred("S", 3, "plus")
    le = t.pred("S", 2, "le")
    val = t.pred("F", 2, "val")
    t.static_init += [(counter, (c,)) for c in cs] + [(value, (v,)) for v in vs]
    t.static_init += [(plus, (vs[a], vs[b], vs[(a + b) % m])) for a in range(m) for b in range(m)]
    t.static_init += [(le, (vs[a], vs[b])) for a in range(m) for b in range(a, m)]
    for c in cs:
        t.fluent_init.append((val, (c, vs[rng.below(m)])))
    t.goal.append((val, True, (cs[0], vs[m - 1])))
    t.schemas.append(("add", 5, [(counter, 1, (0,)), (counter, 1, (1,)), (val, 1, (0, 2)), (val, 1, (1, 3)),
                                 (plus, 1, (2, 3, 4))],
                      [(val, 0, (0, 2)), (val, 1, (0, 4))]))
    t.schemas.append(("double", 3, [(counter, 1, (0,)), (val, 1, (0, 1)), (plus, 1, (1, 1, 2))],
                      [(val, 0, (0, 1)), (val, 1, (0, 2))]))
    t.schemas.append(("reset", 2, [(counter, 1, (0,)), (val, 1, (0, 1)), (le, 1, (1, 1))],
                      [(val, 0, (0, 1)), (val, 1, (0, obj(vs[0])))]))
    return t.text()


CONFIGS = {
    "tower7": lambda: tower(7, 0),
    "transport": lambda: transport(2, 40, 2, 0),
    "tile4x4": lambda: sliding_tile(4, 4, 60, 0),
    "random": lambda: random_domain(0),
}


# ------------------------------------------------------------------------------------------------ random state batches
_K_GOLDEN = -7046029254386353131   # 0x9E3779B97F4A7C15 as int64
_K_MIX1 = -4658895280553007687     # 0xBF58476D1CE4E5B9
_K_MIX2 = -7723592293110705685     # 0x94D049BB133111EB


def _srl(x, k: int):
    """Logical right shift of int64 tensor bits."""
    return (x >> k) & ((1 << (64 - k)) - 1)


def _mix64(x):
    """splitmix64's finalizer on int64 tensors (wrapping multiplies, logical shifts)."""
    x = x ^ _srl(x, 30)
    x = x * _K_MIX1
    x = x ^ _srl(x, 27)
    x = x * _K_MIX2
    return x ^ _srl(x, 31)


def bernoulli_rows(n: int, words: int, slots: int, density: float = 0.05, seed: int = 0, device="cpu",
                   first: int = 0, chunk: int = 1 << 14):
    """A batch of n state rows [n, words] (int64 tensor holding the uint64 words) in which each of the first `slots`
    slots is set independently with probability `density`; slot j of state i is decided by a counter-based draw keyed
    (seed, first + i, j): splitmix64 of seed * golden + (first + i) * 2^20 + j, set iff its top 24 bits are below
    round(density * 2^24). The same (seed, state, slot) always gives the same bit, on any device and in any chunking
    (the successor-generation stress workload draws its 1,048,576 states at 5 % density over every fluent slot)."""
    import torch

    if slots > (1 << 20) or words * 64 < slots:
        raise ValueError("bernoulli_rows: slots must fit the words and be below 2^20")
    thr = int(round(density * (1 << 24)))
    out = torch.zeros((n, words), dtype=torch.int64, device=device)
    j = torch.arange(words * 64, dtype=torch.int64, device=device)
    live = j < slots
    shifts = torch.arange(64, dtype=torch.int64, device=device)
    base_seed = (seed * _K_GOLDEN) & ((1 << 63) - 1)
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        i = torch.arange(first + c0, first + c1, dtype=torch.int64, device=device)
        key = base_seed + (i[:, None] << 20) + j[None, :]
        bits = (_srl(_mix64(key), 40) < thr) & live[None, :]
        out[c0:c1] = (bits.view(c1 - c0, words, 64).to(torch.int64) << shifts).sum(-1)
    return out
