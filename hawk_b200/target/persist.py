"""The persistent entry of an automatic stepping kernel (``<name>_persist``).

An automatic kernel (``steps="auto"``, hawk/trace/steps.py) runs, per sample,
up to ``fused_steps`` trips of its step until the sample finishes.  Trip
counts differ from sample to sample, so a one-sample-per-thread launch keeps a
warp busy until its slowest lane ends.  The persistent entry keeps every lane
busy instead: a resident grid whose lanes take samples off a claim counter,
run each to its finish or its trip budget, write it back and take the next.

Per sample it runs exactly the texts the fused entry runs -- the renderer's
own cut of the fused body (``render_lane_split``, hawk/emit/render.py:153-200:
the head up to the loop, one trip, the tail after it) -- so a sample's planes
hold the same bits as after one fused launch with the same word, whichever
lane runs it and when.  The entry's ABI is the reference's persistent entry's
(hawk/emit/cuda.py:464-520): the kernel's own parameters, then

* ``hawk_next``    uint32 claim counter, zeroed by the caller;
* ``hawk_util``    two uint64 (steps run, lane slots offered) or null;
* ``hawk_steps``   uint32, atomically maxed with the longest per-sample trip
  count, or null;
* ``hawk_stepsum`` uint64, the steps run, or null;
* ``hawk_chunk``   trips between two claims (0: each sample runs whole).

and, as there, a sample finished on entry counts into the finished counter
with the ones finishing in the launch, so the counter (zeroed before the
launch) holds the batch's finished count afterwards.

The b200 loop (one 256-thread block per resident slot, any grid):

1. *claim*: the warp's lanes that hold no sample vote (one ballot); the
   lowest of them adds their number to ``hawk_next`` (one atomic per warp)
   and shuffles the first index out; each takes first + its rank.  A lane
   whose claim falls past ``count`` stops claiming.  A claimed sample not
   finished on entry runs the head: its carried values and live-ins move
   into the lane's registers.
2. *chunk*: up to ``hawk_chunk`` trips of the step, each lane predicated on
   holding a sample; a lane whose sample exits or spends its budget writes
   it back (the tail) and idles until the next claim.  The chunk ends early
   once no lane holds a sample (a warp-uniform vote).
3. the warp leaves once none of its lanes holds a sample or can claim one,
   and reports its longest trip count, its steps and its finished count with
   one warp reduction and one atomic each.

Nothing collective runs inside the step; trip counts, budgets and claims are
32-bit (the host refuses a count of 2^31 samples or more).
"""

from __future__ import annotations

from ..errors import HawkError
from .writer import B200_WRITER, body_text

#: The parameters the contiguous-range entry takes after the kernel's own
#: (hawk/emit/cuda.py:275-279): the longest per-sample trip count and the
#: steps run, each null when not reported.
RANGE_PARAMS = ("unsigned int* hawk_steps", "unsigned long long* hawk_stepsum")

RANGE_SUFFIX = "_range"

#: The parameters the persistent entry takes after the kernel's own.
PERSIST_PARAMS = ("unsigned int* hawk_next", "unsigned long long* hawk_util", "unsigned int* hawk_steps",
                  "unsigned long long* hawk_stepsum", "unsigned int hawk_chunk")

SUFFIX = "_persist"


def _carry_type(ttype) -> str:
    from hawk.emit.spelling import carry_type
    return body_text(carry_type(ttype))


def step_fp64_ops(kernel) -> int | None:
    """The 64-bit floating-point operations of one step of an automatic kernel
    (the renderer's count, ``LaneSplit.fp64_ops``), else ``None``."""
    from hawk.emit.render import render_lane_split

    if getattr(kernel, "one_step", None) is None or getattr(kernel.walk, "finish", None) is None:
        return None
    split = render_lane_split(kernel.sinks, kernel.walk, kind=getattr(kernel, "kind", None), writer=B200_WRITER)
    return None if split is None else int(split.fp64_ops)


def persist_entry(kernel, name: str, wrapper) -> str | None:
    """The text of ``<name>_persist`` for an automatic kernel, else ``None``."""
    from hawk.emit.render import render_lane_split
    from hawk.emit.spelling import binding_name

    walk = kernel.walk
    finish = getattr(walk, "finish", None)
    if getattr(kernel, "one_step", None) is None or finish is None:
        return None
    split = render_lane_split(kernel.sinks, walk, indent="                        ",
                              kind=getattr(kernel, "kind", None), writer=B200_WRITER)
    if split is None or split.count is None:
        raise HawkError(f"{name!r}: its fused body does not cut into head, trip and tail; "
                        "the persistent entry is not built for it")
    counter = binding_name("lookup", _counter_name(kernel))
    finish_call = f"hawk_abi::finish_count({counter});"
    pre, step, post = body_text(split.pre), body_text(split.step), body_text(split.post)
    if post.count(finish_call) != 1:
        raise HawkError(f"{name!r}: its tail does not count its finish once; the persistent entry is not built")
    post = post.replace(finish_call, "++hk_fin;")
    guard = body_text(split.guard) if split.guard is not None else "false"

    carries = [(f"hk_c{j}", _carry_type(t), cname, body_text(init), nxt)
               for j, (cname, t, init, nxt) in enumerate(split.carries)]
    lives = [(f"hk_l{m}", _carry_type(t), lname) for m, (lname, t) in enumerate(split.live_ins)]

    def held(indent: str) -> list:
        return ([f"{indent}const {ct} {cname} = {reg};" for reg, ct, cname, _i, _n in carries]
                + [f"{indent}(void){cname};" for _r, _c, cname, _i, _n in carries])

    head = wrapper.entry_signature(walk, name)
    assert head.endswith("    long long nSamples)")
    head = head[:-1] + ",\n" + ",\n".join(f"    {p}" for p in PERSIST_PARAMS) + ")"
    head = head.replace(f" {name}(", f" {name}{SUFFIX}(", 1)
    p16, p20, p24 = " " * 16, " " * 20, " " * 24
    commit = [*held(p24), post.rstrip("\n"),
              f"{p24}hk_longest = hk_trip > hk_longest ? hk_trip : hk_longest;",
              f"{p24}hk_ran += hk_trip;",
              f"{p24}hk_has = false;"]
    lines = [
        head,
        "{",
        wrapper.unpack(walk),
        *[f"    {ct} {reg}{{}};" for reg, ct, _c, _i, _n in carries],
        *[f"    {lt} {reg}{{}};" for reg, lt, _l in lives],
        "    bool hk_has = false;              // the lane holds a sample with trips left",
        "    bool hk_dry = false;              // the lane's last claim fell past count",
        "    unsigned hk_s = 0u, hk_trip = 0u, hk_budget = 0u, hk_longest = 0u, hk_fin = 0u;",
        "    unsigned long long hk_ran = 0ull;",
        "    const unsigned hk_lane = threadIdx.x & 31u;",
        "    const unsigned hk_chunk = hawk_chunk != 0u ? hawk_chunk : 0xffffffffu;",
        "    (void)nSamples;",
        "    while (true) {",
        "        // claim: the lanes holding no sample take the next ones, one atomic per warp",
        "        const bool hk_needy = !hk_has && !hk_dry;",
        "        const unsigned hk_need = __ballot_sync(0xffffffffu, hk_needy);",
        "        if (hk_need != 0u) {",
        "            const int hk_lead = __ffs(hk_need) - 1;",
        "            unsigned hk_first = 0u;",
        "            if (hk_lane == static_cast<unsigned>(hk_lead))",
        "                hk_first = atomicAdd(hawk_next, static_cast<unsigned>(__popc(hk_need)));",
        "            hk_first = __shfl_sync(0xffffffffu, hk_first, hk_lead);",
        "            if (hk_needy) {",
        "                hk_s = hk_first + static_cast<unsigned>(__popc(hk_need & ((1u << hk_lane) - 1u)));",
        "                if (static_cast<long long>(hk_s) >= count) {",
        "                    hk_dry = true;",
        "                } else {",
        "                    const hk::SampleIndex i{base + static_cast<long long>(hk_s)};",
        f"                    if ({guard}) {{",
        "                        ++hk_fin;             // finished on entry: part of the batch's count",
        "                    } else {",
        pre.rstrip("\n"),
        *[f"{p24}{reg} = {init};" for reg, _ct, _c, init, _n in carries],
        *[f"{p24}{reg} = {lname};" for reg, _lt, lname in lives],
        f"{p24}hk_budget = static_cast<unsigned>(hawk_clamp_count({body_text(split.count)}));",
        f"{p24}hk_trip = 0u;",
        f"{p24}hk_has = true;",
        f"{p24}if (hk_budget == 0u) {{",
        *[("    " + ln if ln.strip() else ln) for ln in commit],
        f"{p24}}}",
        "                    }",
        "                }",
        "            }",
        "        }",
        "        // leave once no lane of the warp holds a sample or can claim one",
        "        if (!__any_sync(0xffffffffu, hk_has || !hk_dry)) break;",
        "        if (!__any_sync(0xffffffffu, hk_has)) continue;",
        "        // the chunk: a lane whose sample ends writes it back and idles until the next claim",
        "        unsigned hk_iter = 0u;",
        "        do {",
        "            if (hk_has) {",
        f"{p16}const hk::SampleIndex i{{base + static_cast<long long>(hk_s)}};",
        f"{p16}(void)i;",
        f"{p16}const int {split.index} = static_cast<int>(hk_trip);",
        f"{p16}(void){split.index};",
        *[f"{p16}const {ct} {cname} = {reg};" for reg, ct, cname, _i, _n in carries],
        *[f"{p16}const {lt} {lname} = {reg};" for reg, lt, lname in lives],
        *[f"{p16}(void){lname};" for _r, _l, lname in lives],
        step.rstrip("\n"),
        *[f"{p16}{reg} = {nxt};" for reg, _ct, _c, _i, nxt in carries],
        f"{p16}++hk_trip;",
        f"{p16}if ({split.exit} || hk_trip >= hk_budget) {{",
        *[ln.replace(p24, p20, 1) if ln.startswith(p24) else ln for ln in commit],
        f"{p16}}}",
        "            }",
        "            ++hk_iter;",
        "        } while (hk_iter < hk_chunk && __any_sync(0xffffffffu, hk_has));",
        "        if (hawk_util != nullptr && hk_lane == 0u) atomicAdd(&hawk_util[1], 32ull * hk_iter);",
        "    }",
        "    // one report per warp: the longest trip count, the steps run, the finished count",
        "    hk::persist_report(hawk_steps, hawk_stepsum, hawk_util, hk_longest, hk_ran);",
        f"    hk::persist_finished({counter}, hk_fin);",
        "}",
    ]
    return "\n".join(lines)


def _counter_name(kernel) -> str:
    """The finished counter's plane name (the sidecar's ``finish.counter``)."""
    from hawk.ir.nodes import FINISHED_PLANE

    return FINISHED_PLANE


def range_entry(kernel, name: str, wrapper) -> str | None:
    """The text of ``<name>_range`` for an automatic kernel, else ``None``.

    The reference's contiguous-range entry (hawk/emit/cuda.py:709-784): the
    kernel's own parameters, then ``hawk_steps`` (uint32, maxed with each
    sample's steps this launch) and ``hawk_stepsum`` (uint64, their sum), each
    null when not reported.  Every sample of ``[base, base + count)`` runs on
    one lane of the grid-stride frame: the word 1 the single step's body (one
    step for a sample not finished on entry), any other word the fused body as
    the renderer cuts it (head, the trips up to the step's exit or the budget,
    tail) -- the texts the persistent entry runs, so the same bits as one
    launch of the kernel's own entry with that word.  A sample finished on
    entry counts into the finished counter with those finishing in the launch.
    Each lane keeps its longest trip count and its steps in registers; one
    warp reduction and one atomic each report them after the frame."""
    from hawk.emit.render import render_body, render_lane_split
    from hawk.emit.spelling import binding_name

    walk = kernel.walk
    one_step = getattr(kernel, "one_step", None)
    if one_step is None or getattr(walk, "finish", None) is None:
        return None
    split = render_lane_split(kernel.sinks, walk, indent="            ",
                              kind=getattr(kernel, "kind", None), writer=B200_WRITER)
    if split is None or split.count is None:
        raise HawkError(f"{name!r}: its fused body does not cut into head, trip and tail; "
                        "the range entry is not built for it")
    from .assemble import _word_read

    counter = binding_name("lookup", _counter_name(kernel))
    on_entry = f"hawk_abi::finish_count({counter});"
    single = body_text(render_body(one_step.sinks, one_step.walk, indent="        ", kind=getattr(kernel, "kind", None),
                                   writer=B200_WRITER).text)
    pre, step, post = body_text(split.pre), body_text(split.step), body_text(split.post)
    guard = body_text(split.guard) if split.guard is not None else None
    carries = [(f"hk_c{j}", _carry_type(t), cname, body_text(init), nxt)
               for j, (cname, t, init, nxt) in enumerate(split.carries)]
    head = wrapper.entry_signature(walk, name)
    assert head.endswith("    long long nSamples)")
    head = head[:-1] + ",\n" + ",\n".join(f"    {p}" for p in RANGE_PARAMS) + ")"
    head = head.replace(f" {name}(", f" {name}{RANGE_SUFFIX}(", 1)
    p12, p16 = " " * 12, " " * 16
    fused = [
        *([f"        if (!({guard})) {{"] if guard is not None else ["        {"]),
        pre.rstrip("\n"),
        *[f"{p12}{ct} {reg} = {init};" for reg, ct, _c, init, _n in carries],
        f"{p12}const int hk_cnt = hawk_clamp_count({body_text(split.count)});",
        f"{p12}unsigned hk_trip = 0u;",
        f"{p12}if (hk_cnt > 0)",
        f"{p12}while (true) {{",
        f"{p16}const int {split.index} = static_cast<int>(hk_trip);",
        f"{p16}(void){split.index};",
        *[f"{p16}const {ct} {cname} = {reg};" for reg, ct, cname, _i, _n in carries],
        step.rstrip("\n"),
        *[f"{p16}{reg} = {nxt};" for reg, _ct, _c, _i, nxt in carries],
        f"{p16}++hk_trip;",
        f"{p16}if ({split.exit} || hk_trip >= static_cast<unsigned>(hk_cnt)) break;",
        f"{p12}}}",
        f"{p12}{{",
        *[f"{p16}const {ct} {cname} = {reg};" for reg, ct, cname, _i, _n in carries],
        *[f"{p16}(void){cname};" for _r, _c, cname, _i, _n in carries],
        post.rstrip("\n"),
        f"{p12}}}",
        f"{p12}hk_longest = hk_trip > hk_longest ? hk_trip : hk_longest;",
        f"{p12}hk_ran += hk_trip;",
        *([f"        }} else {{ {on_entry} }}"] if guard is not None else ["        }"]),
    ]
    lines = [
        head,
        "{",
        wrapper.unpack(walk),
        "    unsigned hk_longest = 0u;",
        "    unsigned long long hk_ran = 0ull;",
        f"    if ({_word_read()} == 1) {{",
        wrapper.index_prologue(),
        f"        const bool hk_live = !({guard});" if guard is not None else "        const bool hk_live = true;",
        single.rstrip("\n"),
        "        if (hk_live) {",
        "            hk_longest = 1u;",
        "            ++hk_ran;",
        *([f"        }} else {{ {on_entry} }}"] if guard is not None else ["        }"]),
        wrapper.index_epilogue(),
        "    } else {",
        wrapper.index_prologue(),
        *fused,
        wrapper.index_epilogue(),
        "    }",
        "    // one report per warp: the longest trip count and the steps run",
        "    hk::persist_report(hawk_steps, hawk_stepsum, nullptr, hk_longest, hk_ran);",
        "}",
    ]
    return "\n".join(line for line in lines if line is not None)
