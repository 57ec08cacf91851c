"""Execution-plan verifier and workspace slot assignment (host only).

The verifier must accept exactly the allocations that are safe: every read
sees a produced buffer, every slot holds its buffers, and two buffers share a
slot only when the later one's producer runs after every access of the earlier
one -- in stream order, or through declared dependency edges in graph mode.
Cases mirror the reference's own plan-verifier tests (tests/cpp/pass.cpp:160-318,
diagnostic texts included); generated plans are checked against an independent
brute-force validity rule written here (pairwise lifetimes, transitive
closure), not against the verifier's adjacent-slot search.  Where the
reference's own PASS checker is built from its sources (oracle/_ref,
oracle/ref_build.py), every verdict and diagnostic is also compared with it.
"""
import itertools
import random

import pytest

from ask_b200 import runtime as rt

BIG = 2 ** 64 - 1


def plan(buffer_count, inputs, outputs, steps):
    return {"buffer_count": buffer_count, "public_inputs": list(inputs), "public_outputs": list(outputs),
            "steps": [{"inputs": list(i), "outputs": list(o)} for i, o in steps]}


def chain(n):
    return plan(n + 1, [0], [n], [([i], [i + 1]) for i in range(n)])


def allocation(p, sizes, assignments, capacities, graph=False, dependencies=None):
    a = dict(p)
    a.update({"buffer_sizes": list(sizes), "assignments": [list(x) for x in assignments],
              "slot_capacity_bytes": list(capacities), "graph": graph})
    if dependencies is not None:
        a["dependencies"] = [list(d) for d in dependencies]
    return a


def _reference():
    from oracle import ref
    return ref if ref.load() is not None else None


REF = _reference()


def check(a):
    """Our verifier; equal to the reference's PASS checker, text included."""
    ours = rt.check_allocation(a)
    if REF is not None:
        assert REF.pass_check(a) == ours, a
    return ours


# ---- the reference's explicit cases ------------------------------------------------
def test_two_slots_for_a_four_step_chain():
    p = chain(4)
    assert check(p) == (True, "")
    assert check(allocation(p, [16] * 5, [(1, 0), (2, 1), (3, 0)], [16, 16]))[0]


def test_passthroughs_and_long_plans():
    p = plan(1, [0], [0], [([], [])] * 299 + [([0], [])])
    assert check(allocation(p, [16], [], []))[0]
    long = chain(150)
    assert check(allocation(long, [16] * 151, [(i, (i - 1) % 2) for i in range(1, 150)], [16, 16]))[0]
    assert check(allocation(plan(1, [0], [0], []), [16], [], []))[0]
    p4 = chain(4)
    assert check(allocation(p4, [16, 0, 0, 0, 16], [(1, 0), (2, 1), (3, 0)], [0, 0]))[0]


def test_diagnostics():
    p = chain(4)
    ok, text = check(allocation(p, [16] * 5, [(1, 0), (2, 0), (3, 0)], [16]))
    assert not ok and "ADJACENT_1_2 FAIL" in text
    ok, text = check(allocation(p, [16] * 5, [(1, 0), (2, 1), (3, 0)], [15, 16]))
    assert not ok and "CAPACITY_1 FAIL" in text
    bad = chain(4)
    bad["steps"][0]["inputs"] = [1]
    ok, text = check(allocation(bad, [16] * 5, [(1, 0), (2, 0), (3, 0)], [15]))
    assert not ok
    assert text == ("verify READ_0_0 FAIL\nverify CAPACITY_1 FAIL\nverify CAPACITY_2 FAIL\n"
                    "verify CAPACITY_3 FAIL\nverify ADJACENT_1_2 FAIL\nverify ADJACENT_2_3 FAIL\n")


@pytest.mark.parametrize("assignments,capacities,message", [
    ([(1, 0), (2, 1)], [16, 16], "internal buffer has no slot assignment"),
    ([(1, 0), (2, 1), (3, 0), (1, 1)], [16, 16], "internal buffer has multiple slot assignments"),
    ([(1, 2), (2, 1), (3, 0)], [16, 16], "allocation assignment index is out of range"),
    ([(1, 0), (2, 1), (3, 0), (4, 0)], [16, 16], "public port cannot use an internal slot"),
    ([(1, 0), (2, 1), (3, 0)], [16, 16, 16], "allocation contains an unused slot"),
])
def test_malformed_mappings(assignments, capacities, message):
    ok, text = check(allocation(chain(4), [16] * 5, assignments, capacities))
    assert not ok and text == message


def test_same_step_writes_cannot_share():
    p = plan(4, [0], [3], [([0], [1, 2]), ([1, 2], [3])])
    assert not check(allocation(p, [16] * 4, [(1, 0), (2, 0)], [16]))[0]


def test_three_lifetimes_in_one_slot_and_a_long_lived_first():
    p = chain(6)
    a = allocation(p, [16] * 7, [(1, 0), (2, 1), (3, 0), (4, 1), (5, 0)], [16, 16])
    assert check(a)[0]
    a["steps"][4]["inputs"].append(1)  # buffer 1 now lives until step 4, overlapping buffer 5's slot mate 3
    assert not check(a)[0]


def test_read_before_write():
    p = chain(4)
    p["steps"][0]["inputs"] = [2]
    ok, text = check(p)
    assert not ok and "READ_0_0" in text


@pytest.mark.parametrize("p,message", [
    (plan(2, [0, 0], [1], [([0], [1])]), "public input buffer is repeated"),
    (plan(2, [0], [1], [([0], [1]), ([0], [1])]), "buffer has multiple writers or aliases a public input"),
    (plan(2, [0], [], [([0], [1])]), "plan must have a public output"),
    (plan(3, [0], [1], [([0], [1])]), "plan contains a buffer without a writer"),
    (plan(2, [0], [5], [([0], [1])]), "public output buffer index is out of range"),
])
def test_structural_errors(p, message):
    assert check(p) == (False, message)


def test_graph_structure_errors():
    p = chain(3)
    base = allocation(p, [16] * 4, [(1, 0), (2, 1)], [16, 16], graph=True, dependencies=[[], [0], [1]])
    assert check(base)[0]
    for deps, message in [([[], [0]], "graph dependency count differs from the plan"),
                          ([[], [1], [1]], "graph dependency is not topologically ordered"),
                          ([[], [0, 0], [1]], "graph dependency is repeated")]:
        a = dict(base, dependencies=deps)
        assert check(a) == (False, message)
    assert check(dict(base, graph=False)) == (False, "stream plan contains graph dependencies")


def test_graph_order_needs_edges_not_index_order():
    # two independent branches: reusing a slot across them needs an edge
    p = plan(5, [0], [3, 4], [([0], [1]), ([0], [2]), ([1], [3]), ([2], [4])])
    a = allocation(p, [16] * 5, [(1, 0), (2, 0)], [16], graph=True, dependencies=[[], [], [0], [1]])
    ok, text = check(a)
    assert not ok and "GRAPH_ORDER_1" in text
    a["dependencies"] = [[], [], [0], [1]]
    a["assignments"] = [[1, 0], [2, 1]]
    a["slot_capacity_bytes"] = [16, 16]
    assert check(a)[0]
    # an ordering edge from the reader of buffer 1 to the producer of buffer 2 makes sharing safe
    p2 = plan(5, [0], [3, 4], [([0], [1]), ([1], [3]), ([0], [2]), ([2], [4])])
    a2 = allocation(p2, [16] * 5, [(1, 0), (2, 0)], [16], graph=True, dependencies=[[], [0], [1], [2]])
    assert check(a2)[0]
    a2["dependencies"][2] = []
    assert not check(a2)[0]


def test_graph_mode_reads_need_a_path_to_their_producer():
    p = chain(3)
    a = allocation(p, [16] * 4, [(1, 0), (2, 1)], [16, 16], graph=True, dependencies=[[], [], [1]])
    ok, text = check(a)
    assert not ok and text == "verify GRAPH_ORDER_1 FAIL\n"


# ---- generated plans against a brute-force rule ------------------------------------
def topology(kind, n):
    if kind == "chain":
        return chain(n)
    if kind == "fork":  # root, then n-1 branches that all read it
        steps = [([0], [1])] + [([1], [i + 1]) for i in range(1, n)]
        return plan(n + 1, [0], list(range(2, n + 1)), steps)
    if kind == "join":  # n-1 independent producers, then one step reading them all
        steps = [([0], [i + 1]) for i in range(n - 1)] + [(list(range(1, n)), [n])]
        return plan(n + 1, [0], [n], steps)
    if kind == "unused":  # scratch-like writes nobody reads
        steps = [([0], [i + 1]) for i in range(n - 1)] + [([0], [n])]
        return plan(n + 1, [0], [n], steps)
    raise ValueError(kind)


def producers(p):
    prod = {}
    for s, step in enumerate(p["steps"]):
        for b in step["outputs"]:
            prod[b] = s
    return prod


def accesses(p):
    acc = {}
    for s, step in enumerate(p["steps"]):
        for b in step["inputs"] + step["outputs"]:
            acc.setdefault(b, set()).add(s)
    return acc


def closure(deps):
    n = len(deps)
    before = [[False] * n for _ in range(n)]
    for s in range(n):
        for d in deps[s]:
            before[d][s] = True
            for x in range(d):
                before[x][s] = before[x][s] or before[x][d]
    return before


def brute_valid(a):
    p = a["plan"] if "plan" in a else a
    prod = producers(a)
    acc = accesses(a)
    born = {b: 0 for b in a["public_inputs"]}
    born.update({b: s + 1 for b, s in prod.items()})
    for s, step in enumerate(a["steps"]):
        if any(born[b] > s for b in step["inputs"]):
            return False
    caps = a["slot_capacity_bytes"]
    if any(a["buffer_sizes"][b] > caps[k] for b, k in a["assignments"]):
        return False
    slot = {}
    for b, k in a["assignments"]:
        slot.setdefault(k, []).append(b)
    n = len(a["steps"])
    if not a.get("graph"):
        for users in slot.values():
            for x, y in itertools.permutations(users, 2):
                if prod[x] <= prod[y] and max(acc[x]) >= prod[y]:
                    return False
        return True
    before = closure(a["dependencies"])
    for s, step in enumerate(a["steps"]):
        for b in step["inputs"]:
            if b in prod and not before[prod[b]][s]:
                return False
    for users in slot.values():
        for x, y in itertools.permutations(users, 2):
            if prod[x] <= prod[y] and not all(t < prod[y] and before[t][prod[y]] for t in acc[x]):
                return False
    return True


@pytest.mark.parametrize("kind", ["chain", "fork", "join", "unused"])
@pytest.mark.parametrize("n", [2, 4, 5])
@pytest.mark.parametrize("delayed_read", [False, True])
def test_stream_mappings_match_brute_force(kind, n, delayed_read):
    p = topology(kind, n)
    if delayed_read and n > 2:
        p["steps"][-1]["inputs"].append(1)
    internal = [b for b in range(p["buffer_count"]) if b not in p["public_inputs"] + p["public_outputs"]]
    for bytes_, short in [(16, False), (16, True), (0, False), (BIG, True)]:
        sizes = [bytes_] * p["buffer_count"]
        for mapping in itertools.product(range(len(internal)), repeat=len(internal)):
            used = sorted(set(mapping))
            if used != list(range(len(used))):
                continue  # slots must be dense
            caps = [bytes_] * len(used)
            if short and bytes_:
                caps[0] -= 1
            a = allocation(p, sizes, list(zip(internal, mapping)), caps)
            assert check(a)[0] == brute_valid(a), (kind, n, mapping, bytes_, short)


@pytest.mark.parametrize("kind", ["chain", "fork", "join", "unused"])
@pytest.mark.parametrize("n", [3, 5])
def test_graph_mappings_match_brute_force(kind, n):
    p = topology(kind, n)
    prod = producers(p)
    data_deps = [sorted({prod[b] for b in step["inputs"] if b in prod}) for step in p["steps"]]
    chain_deps = [sorted(set(d) | ({s - 1} if s else set())) for s, d in enumerate(data_deps)]
    internal = [b for b in range(p["buffer_count"]) if b not in p["public_inputs"] + p["public_outputs"]]
    rng = random.Random(n * 31 + len(kind))
    for deps in (data_deps, chain_deps):
        for mapping in itertools.product(range(len(internal)), repeat=len(internal)):
            used = sorted(set(mapping))
            if used != list(range(len(used))):
                continue
            a = allocation(p, [16] * p["buffer_count"], list(zip(internal, mapping)), [16] * len(used), True, deps)
            assert check(a)[0] == brute_valid(a), (kind, n, deps, mapping)
        # random edge mutations of a valid plan: drop, repeat, reverse
        for _ in range(20):
            d = [list(x) for x in deps]
            s = rng.randrange(1, len(d))
            if d[s]:
                j = rng.randrange(len(d[s]))
                op = rng.randrange(3)
                if op == 0:
                    d[s].pop(j)
                elif op == 1:
                    d[s].append(d[s][j])
                else:
                    d[s][j] = s
            a = allocation(p, [16] * p["buffer_count"], [(b, k) for k, b in enumerate(internal)], [16] * len(internal),
                           True, d)
            assert (check(a)[0]) == (valid_deps(d) and brute_valid(a))


def valid_deps(deps):
    return all(x < s for s, d in enumerate(deps) for x in d) and all(len(set(d)) == len(d) for d in deps)


# ---- slot assignment ---------------------------------------------------------------
@pytest.mark.parametrize("kind", ["chain", "fork", "join", "unused"])
@pytest.mark.parametrize("n", [2, 3, 6, 40])
@pytest.mark.parametrize("graph", [False, True])
def test_assigned_slots_verify(kind, n, graph):
    p = topology(kind, n)
    sizes = [(7 * b) % 5 * 16 for b in range(p["buffer_count"])]
    out = rt.assign_slots(dict(p, buffer_sizes=sizes), graph)
    a = dict(p, buffer_sizes=sizes, **out)
    assert check(a) == (True, "")
    assert brute_valid(a)


def test_slot_counts():
    # four serial steps have three internal buffers; two slots suffice in either mode
    for graph in (False, True):
        out = rt.assign_slots(dict(chain(4), buffer_sizes=[16] * 5), graph)
        assert len(out["slot_capacity_bytes"]) == 2
    # unread writes are live only at their producer: one slot in stream order,
    # one per step in graph order (no edge orders independent producers)
    p = topology("unused", 5)
    assert len(rt.assign_slots(dict(p, buffer_sizes=[16] * 6), False)["slot_capacity_bytes"]) == 1
    assert len(rt.assign_slots(dict(p, buffer_sizes=[16] * 6), True)["slot_capacity_bytes"]) == 4
    # a long chain reuses two slots; its graph has one edge per step after the first
    out = rt.assign_slots(dict(chain(2000), buffer_sizes=[16] * 2001), True)
    assert len(out["slot_capacity_bytes"]) == 2
    assert sum(len(d) for d in out["dependencies"]) == 1999


def test_capacity_is_the_largest_occupant():
    p = chain(5)
    sizes = [4, 100, 8, 300, 2, 4]
    out = rt.assign_slots(dict(p, buffer_sizes=sizes), False)
    caps = out["slot_capacity_bytes"]
    for b, k in out["assignments"]:
        assert sizes[b] <= caps[k]
    assert sorted(caps) == [8, 300]  # slot 0 holds buffers 1 and 3, slot 1 holds 2 and 4


def test_reference_pass_checker_was_compared():
    """The comparisons above ran against the reference's PASS (when built)."""
    if REF is None:
        pytest.skip("the reference's PASS checker is not built here (oracle/_ref)")
    ok, text = REF.pass_check(chain(4))
    assert ok and text == ""


# ---- random plans, defects included, against the reference's checker -----------------
def _random_allocation(rng):
    """A random plan, mapping and (in graph mode) edge list.  Roughly half are
    built valid and then perturbed once: a buffer moved to another slot, a
    capacity cut, an edge dropped or a structural defect (bad index, second
    writer, unused slot, public buffer in a slot)."""
    nsteps = rng.randint(1, 9)
    nin = rng.randint(1, 3)
    bufs = nin
    steps = []
    for s in range(nsteps):
        reads = rng.sample(range(bufs), rng.randint(1, min(3, bufs)))
        writes = list(range(bufs, bufs + rng.randint(1, 2)))
        bufs += len(writes)
        steps.append((reads, writes))
    outputs = sorted(rng.sample(range(nin, bufs), rng.randint(1, min(2, bufs - nin))))
    p = plan(bufs, range(nin), outputs, steps)
    graph = rng.random() < 0.5
    sizes = [rng.choice([0, 8, 16, 64]) for _ in range(bufs)]
    out = rt.assign_slots(dict(p, buffer_sizes=sizes), graph)
    a = dict(p, buffer_sizes=sizes, **out)
    a["assignments"] = [list(x) for x in a["assignments"]]
    kind = rng.randrange(9)
    if kind == 0 and len(a["slot_capacity_bytes"]) > 1 and a["assignments"]:
        e = rng.choice(a["assignments"])
        e[1] = rng.randrange(len(a["slot_capacity_bytes"]))
    elif kind == 1 and a["slot_capacity_bytes"]:
        k = rng.randrange(len(a["slot_capacity_bytes"]))
        a["slot_capacity_bytes"][k] = max(0, a["slot_capacity_bytes"][k] - 8)
    elif kind == 2 and graph:
        deps = [d for d in a["dependencies"] if d]
        if deps:
            d = rng.choice(deps)
            d.pop(rng.randrange(len(d)))
    elif kind == 3:
        st = rng.choice(a["steps"])
        st[rng.choice(["inputs", "outputs"])].append(rng.choice([bufs, bufs + 3, 0]))
    elif kind == 4:
        a["slot_capacity_bytes"].append(16)
    elif kind == 5 and a["assignments"]:
        a["assignments"].append([rng.choice(outputs), 0])
    elif kind == 6:
        rng.shuffle(a["steps"])
        if graph:
            a["dependencies"] = [[x for x in d if x < s] for s, d in enumerate(a["dependencies"])]
    elif kind == 7:
        a["public_outputs"] = [] if rng.random() < 0.5 else [bufs + 1]
    return a


@pytest.mark.skipif(REF is None, reason="the reference's PASS checker is not built here (oracle/_ref)")
def test_random_allocations_match_the_reference_checker():
    rng = random.Random(0xA5C)
    verdicts = set()
    for _ in range(3000):
        a = _random_allocation(rng)
        ours = rt.check_allocation(a)
        assert REF.pass_check(a) == ours, a
        verdicts.add(ours[0])
    assert verdicts == {True, False}
