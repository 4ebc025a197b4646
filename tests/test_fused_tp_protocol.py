"""Model check of the fused tensor-parallel boundary protocol (buffer reuse, epochs and
programmatic dependent launch), on CPU.

Every rank runs the same kernel sequence per forward (parallel.fused_tp,
models/decoder.py `_forward_fused_tp`):

    START(0)  [ GAG(2l) ATT GRS(2l+1) RSN(2l+1) GAG(2l+1) GRS(2l+2) RSN(2l+2) ]*L  LOGITS  END

  GRS(c)  reduce-scatter GEMM: writes this rank's slot on every owner, then releases
          the owners' RS flags of call c                      (normal launch)
  RSN(c)  waits for the RS flags of call c from every rank, reads its own slots,
          writes its rows into every rank's gather buffer, releases AG flags
          (programmatic dependent of the previous kernel)
  START   writes the embedding rows into every gather buffer, releases AG flags (normal)
  GAG(c)  waits for the AG flags of call c, reads the local gather buffer
          (programmatic dependent)
  ATT     attention between QKV and o_proj (normal); LOGITS waits for the AG flags of
          the final call (`FusedTP.wait_gathered`) and reads the final gather rows, and
          the logits all-gather is a collective: no rank starts the next forward before
          every rank's LOGITS finished.

Launch semantics: a normal kernel starts after its predecessor on the rank completed;
a programmatic dependent starts once its predecessor started (every CTA triggers on
entry) and completes only after it (griddepcontrol.wait before exit).  Flags carry
epochs (step * 256 + call + 1) and waits are `>=`.

A random scheduler fires enabled actions (start, each rank-region read, each write,
each flag release, completion) in random orders; the checker asserts that no slot or
gather region is written with a new version while a reader that needs the previous
version has not read it yet, and that every read sees the version it waited for.
"""
import random

import pytest

NORMAL, PDL = 0, 1


def _program(L, grs_launch=NORMAL, rsn_launch=PDL, gag_launch=PDL):
    prog = [("START", 0, NORMAL)]
    for layer in range(L):
        prog.append(("GAG", 2 * layer, gag_launch))
        prog.append(("ATT", None, NORMAL))
        for c in (2 * layer + 1, 2 * layer + 2):
            prog.append(("GRS", c, grs_launch))
            prog.append(("RSN", c, rsn_launch))
            if c == 2 * layer + 1:
                prog.append(("GAG", c, gag_launch))
    prog.append(("LOGITS", 2 * L, NORMAL))
    prog.append(("END", None, NORMAL))
    return prog


class Violation(AssertionError):
    pass


def simulate(W, L, steps, seed, logits_waits=True, **launch):
    rng = random.Random(seed)
    prog = _program(L, **launch)
    n = len(prog)
    # buffer versions: slot[o][src], gather[d][o] hold (step, call) of their last write
    slot = {(o, s): None for o in range(W) for s in range(W)}
    gather = {(d, o): None for d in range(W) for o in range(W)}
    rs_flag = {(o, s): -1 for o in range(W) for s in range(W)}    # epoch released by src for owner o
    ag_flag = {(d, o): -1 for d in range(W) for o in range(W)}    # epoch released by owner o on rank d
    # per rank: position in the program, per kernel instance its phase state
    state = {}          # (rank, step, idx) -> the started kernel: reads / writes / flags left, done
    pos = {r: (0, 0) for r in range(W)}        # next kernel to start: (step, idx)
    logits_done = {s: set() for s in range(steps)}

    def ep(step, c):
        return step * 256 + c + 1

    def kernel(r, step, i):
        return state.get((r, step, i))

    def prev_done(r, step, i):
        if i == 0:
            if step == 0:
                return True
            return (kernel(r, step - 1, n - 1) or {}).get("done", False)
        return (kernel(r, step, i - 1) or {}).get("done", False)

    def prev_started(r, step, i):
        if i == 0:
            return prev_done(r, step, i)
        return kernel(r, step, i - 1) is not None

    def can_start(r):
        step, i = pos[r]
        if step >= steps:
            return False
        name, c, mode = prog[i]
        if name == "START" and step > 0 and len(logits_done[step - 1]) < W:
            return False                       # logits all-gather of the previous forward
        return prev_done(r, step, i) if mode == NORMAL else prev_started(r, step, i)

    def start(r):
        step, i = pos[r]
        name, c, mode = prog[i]
        k = {"name": name, "c": c, "mode": mode, "done": False}
        if name == "GRS":
            k["writes"] = [("slot", (o, r)) for o in range(W)]
            k["flags"] = [("rs", (o, r)) for o in range(W)]
        elif name == "RSN":
            k["reads"] = [("slot", (r, s)) for s in range(W)]
            k["writes"] = [("gather", (d, r)) for d in range(W)]
            k["flags"] = [("ag", (d, r)) for d in range(W)]
        elif name == "START":
            k["writes"] = [("gather", (d, r)) for d in range(W)]
            k["flags"] = [("ag", (d, r)) for d in range(W)]
        elif name in ("GAG", "LOGITS"):
            k["reads"] = [("gather", (r, o)) for o in range(W)]
        for key in ("reads", "writes", "flags"):
            k.setdefault(key, [])
        state[(r, step, i)] = k
        pos[r] = (step, i + 1) if i + 1 < n else (step + 1, 0)

    def ready_reads(r, step, k):
        """A read may happen once its guarding flag carries this call's epoch."""
        out = []
        for kind, key in k["reads"]:
            if kind == "slot":
                o, s = key
                if rs_flag[(o, s)] >= ep(step, k["c"]):
                    out.append((kind, key))
            else:
                d, o = key
                if (k["name"] == "LOGITS" and not logits_waits) or ag_flag[(d, o)] >= ep(step, k["c"]):
                    out.append((kind, key))
        return out

    def check_read(step, k, kind, key):
        buf = slot if kind == "slot" else gather
        want = (step, k["c"])
        if buf[key] != want:
            raise Violation(f"{k['name']}({k['c']}) step {step} read {kind}{key} at version {buf[key]}, want {want}")

    def write(step, k, kind, key):
        buf = slot if kind == "slot" else gather
        cur = buf[key]
        if cur is not None:
            # every reader of the current version must have read it already
            s_cur, c_cur = cur
            readers_needed = {"slot": ("RSN",), "gather": ("GAG", "LOGITS")}[kind]
            owner_rank = key[0]
            for i, (name, c, _) in enumerate(prog):
                if name in readers_needed and c == c_cur:
                    kk = kernel(owner_rank, s_cur, i)
                    if kk is None or (kind, key) in kk["reads"]:
                        raise Violation(f"{k['name']}({k['c']}) step {step} overwrote {kind}{key} version {cur} "
                                        f"before {name}({c}) on rank {owner_rank} read it")
        buf[key] = (step, k["c"])

    while True:
        actions = []
        for r in range(W):
            if can_start(r):
                actions.append(("start", r, None))
        for (r, step, i), k in state.items():
            if k["done"]:
                continue
            for rd in ready_reads(r, step, k):
                actions.append(("read", (r, step, i), rd))
            if not k["reads"]:
                for w in k["writes"]:
                    actions.append(("write", (r, step, i), w))
                if not k["writes"]:
                    for f in k["flags"]:
                        actions.append(("flag", (r, step, i), f))
                    if not k["flags"]:
                        pre_ok = True
                        if k["mode"] == PDL and i > 0:
                            pre_ok = kernel(r, step, i - 1)["done"]
                        if pre_ok:
                            actions.append(("done", (r, step, i), None))
        if not actions:
            break
        kind, who, what = rng.choice(actions)
        if kind == "start":
            start(who)
            continue
        r, step, i = who
        k = state[who]
        if kind == "read":
            check_read(step, k, *what)
            k["reads"].remove(what)
        elif kind == "write":
            write(step, k, *what)
            k["writes"].remove(what)
        elif kind == "flag":
            fk, key = what
            (rs_flag if fk == "rs" else ag_flag)[key] = ep(step, k["c"])
            k["flags"].remove(what)
        else:
            k["done"] = True
            if k["name"] == "LOGITS":
                logits_done[step].add(r)
    unfinished = [(key, k["name"]) for key, k in state.items() if not k["done"]]
    if unfinished or any(pos[r][0] < steps for r in range(W)):
        raise Violation(f"deadlock: unfinished kernels {unfinished[:4]}, positions {pos}")


@pytest.mark.parametrize("W", [2, 3, 4])
def test_fused_tp_protocol_has_no_reuse_race(W):
    for seed in range(150):
        simulate(W, L=2, steps=3, seed=seed)


def test_model_catches_a_programmatic_reduce_scatter_launch():
    """Launching the reduce-scatter GEMM as a programmatic dependent too would let a rank
    overwrite an owner's slot before the owner's add+RMSNorm read the previous call; the
    model must find such an interleaving."""
    with pytest.raises(Violation):
        for seed in range(400):
            simulate(2, L=2, steps=2, seed=seed, grs_launch=PDL)


def test_model_catches_an_lm_head_that_does_not_wait_for_the_final_gather():
    """Without the wait on the final boundary's all-gather flags the LM head can read a
    row another owner has not stored yet (the previous forward's version)."""
    with pytest.raises(Violation):
        for seed in range(400):
            simulate(2, L=1, steps=3, seed=seed, logits_waits=False)
