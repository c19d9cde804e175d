"""Pipeline schedules: per-stage action lists for P stages and M microbatches.

An action is ``("F", m)`` forward, ``("B", m)`` backward (input and weight gradients together), or for
zero-bubble schedules ``("B", m)`` input gradient only plus a later ``("W", m)`` weight gradient.

* ``gpipe``: every forward, then every backward (sync GPipe, megagpt-speedrun/sync_pipeline.py:80-216).
* ``one_f_one_b``: ``P - s - 1`` warm-up forwards on stage ``s``, then alternating F/B, then the
  remaining backwards (the standard non-interleaved 1F1B).
* ``zb_h1``: the zero-bubble ZB-H1 order from a greedy wavefront simulation in which every stage, at
  every unit tick, runs the highest-priority ready action with priority B > F > W and at most
  ``P - s`` forwards in flight (1F1B's activation memory); W actions fill the bubbles
  (grug-moe-pp/pipeline_zb.py:325-416 describes the same rule).

``simulate(schedule, t_f, t_b, t_w)`` replays a schedule with per-action costs and cross-stage
dependencies and returns the makespan and bubble fraction.
"""

from __future__ import annotations

Action = tuple[str, int]


def gpipe(P: int, M: int) -> list[list[Action]]:
    return [[("F", m) for m in range(M)] + [("B", m) for m in range(M)] for _ in range(P)]


def one_f_one_b(P: int, M: int) -> list[list[Action]]:
    out = []
    for s in range(P):
        warm = min(P - s - 1, M)
        acts = [("F", m) for m in range(warm)]
        f, b = warm, 0
        while f < M:
            acts.append(("F", f))
            f += 1
            acts.append(("B", b))
            b += 1
        while b < M:
            acts.append(("B", b))
            b += 1
        out.append(acts)
    return out


def zb_h1(P: int, M: int, t_f: int = 1, t_b: int = 1, t_w: int = 1, w_slack: int = 1) -> list[list[Action]]:
    """Greedy wavefront with integer action costs; returns each stage's action order.

    A microbatch's activations stay alive until its W (the weight gradient reads them), so a stage
    starts a new forward only while fewer than ``P - s + w_slack`` microbatches lack their W: the
    deferred W passes fill bubbles, but never hold more activations than 1F1B does plus ``w_slack``
    microbatches (without the bound a stage with no bubbles would defer every W to the end)."""
    done: dict[tuple[str, int, int], int] = {}  # (kind, stage, mb) -> finish time
    nxt_f = [0] * P
    nxt_b = [0] * P
    w_done = [0] * P
    pending_w: list[list[int]] = [[] for _ in range(P)]
    busy_until = [0] * P
    order: list[list[Action]] = [[] for _ in range(P)]
    cost = {"F": t_f, "B": t_b, "W": t_w}
    total = 3 * P * M
    t = 0
    while sum(len(o) for o in order) < total:
        for s in range(P):
            if busy_until[s] > t:
                continue
            choice = None
            m = nxt_b[s]
            if m < nxt_f[s]:
                dep = done.get(("B", s + 1, m)) if s + 1 < P else done.get(("F", s, m))
                if dep is not None and dep <= t:
                    choice = ("B", m)
            if (choice is None and nxt_f[s] < M and nxt_f[s] - nxt_b[s] < P - s
                    and nxt_f[s] - w_done[s] < P - s + w_slack):
                m = nxt_f[s]
                dep = done.get(("F", s - 1, m)) if s > 0 else 0
                if dep is not None and dep <= t:
                    choice = ("F", m)
            if choice is None and pending_w[s]:
                choice = ("W", pending_w[s][0])
            if choice is None:
                continue
            k, m = choice
            if k == "F":
                nxt_f[s] += 1
            elif k == "B":
                nxt_b[s] += 1
                pending_w[s].append(m)
            else:
                pending_w[s].pop(0)
                w_done[s] += 1
            order[s].append(choice)
            busy_until[s] = t + cost[k]
            done[(k, s, m)] = t + cost[k]
        t += 1
        if t > 100 * total * max(cost.values()):
            raise RuntimeError("schedule simulation did not converge")
    return order


def simulate(schedule: list[list[Action]], t_f: float = 1.0, t_b: float = 2.0, t_w: float | None = None):
    """Replay with costs (``t_b`` is the full backward when the schedule has no W actions, the input
    gradient alone otherwise). Returns ``{"makespan", "bubble"}``."""
    P = len(schedule)
    split = any(k == "W" for acts in schedule for k, _ in acts)
    tw = (t_w if t_w is not None else 0.0) if split else 0.0
    cost = {"F": t_f, "B": t_b, "W": tw}
    fin: dict[tuple[str, int, int], float] = {}
    pos = [0] * P
    clock = [0.0] * P
    remaining = sum(len(a) for a in schedule)
    while remaining:
        progressed = False
        for s in range(P):
            if pos[s] >= len(schedule[s]):
                continue
            k, m = schedule[s][pos[s]]
            if k == "F":
                dep = fin.get(("F", s - 1, m)) if s > 0 else 0.0
            elif k == "B":
                dep = fin.get(("B", s + 1, m)) if s + 1 < P else fin.get(("F", s, m))
            else:
                dep = fin.get(("B", s, m))
            if dep is None:
                continue
            start = max(clock[s], dep)
            clock[s] = start + cost[k]
            fin[(k, s, m)] = clock[s]
            pos[s] += 1
            remaining -= 1
            progressed = True
        if not progressed:
            raise RuntimeError("schedule deadlocks")
    makespan = max(clock)
    work = sum(cost[k] for acts in schedule for k, _ in acts)
    return {"makespan": makespan, "bubble": 1.0 - work / (P * makespan)}


SCHEDULES = {"gpipe": gpipe, "1f1b": one_f_one_b, "zb": zb_h1}


def validate(schedule: list[list[Action]], M: int) -> None:
    """Every stage runs each microbatch's F and B once (and W once if any), B after F, W after B."""
    for s, acts in enumerate(schedule):
        seen = set()
        for k, m in acts:
            if (k, m) in seen:
                raise ValueError(f"stage {s}: {k}{m} twice")
            if k == "B" and ("F", m) not in seen:
                raise ValueError(f"stage {s}: B{m} before F{m}")
            if k == "W" and ("B", m) not in seen:
                raise ValueError(f"stage {s}: W{m} before B{m}")
            seen.add((k, m))
        for m in range(M):
            if ("F", m) not in seen or ("B", m) not in seen:
                raise ValueError(f"stage {s}: microbatch {m} incomplete")
