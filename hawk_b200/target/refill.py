"""The lane-refill frame: a body with one data-dependent loop, its lanes kept busy.

A per-sample loop with a ``break`` (Kepler's Newton solve: 3 to 7 trips)
runs, in the lane frame, as long as the warp's slowest lane: the lanes whose
sample has left idle until then.  This frame runs the same body cut at its
loop -- the renderer's own texts for the head before the loop, one trip, and
the tail after it (``render_lane_segments``, hawk/emit/render.py:302; the cut
the reference's host target interchanges, hawk/ir/vectorise.py:64) -- with each
lane holding one sample's carried values in registers: a lane whose sample
leaves the loop runs its tail (the commits) and takes the next sample at once.

Work is claimed without atomics.  Warp w of W owns the spans of 32 R
consecutive samples starting at (w + k W) * 32 R, k = 0, 1, ...; the lanes
that need a sample vote (one ballot) and take the next ones of the warp's
current span in lane order, every lane keeping the same span cursor.  A warp
leaves once no lane holds a sample and its next span starts past ``count``.
(Holding a second sample per lane, its head run ahead so its loads overlap the
trips, measured slower for Kepler: 1.228 against 1.197 ms at 2^24.)

Each sample runs exactly the plain body's operations, so the planes hold the
same bits as with the lane frame, whatever lane runs a sample and when.
Admitted: no sample sums, one top-level loop counted from 0 by 1 to a static
bound, with a ``break``; every value the trip or the tail reads from the head
a one-line declaration of a known type.
"""

from __future__ import annotations

import re

from .writer import B200_WRITER, body_text

#: Spans of 32 * SPAN_ROWS samples per warp claim.  Kepler at 2^20 / 2^24
#: samples: 0.0861 / 1.192 ms with spans of 64, 0.0957 / 1.196 ms with 256
#: (the lane frame: 0.0911 / 1.349 ms).
SPAN_ROWS = 2

_DECL = re.compile(r"^\s*const auto (\w+) = ")
_WORD = re.compile(r"\b[A-Za-z_]\w*\b")


def refill_frame(kernel, walk) -> str | None:
    """The entry's frame and body text under lane refill, else ``None``."""
    from hawk.emit.render import render_lane_segments
    from hawk.emit.spelling import carry_type
    from hawk.ir.vectorise import interchanged_loops

    cut = interchanged_loops(walk)
    if len(cut) != 1:
        return None
    seg = render_lane_segments(kernel.sinks, walk, cut, indent="            ", kind=getattr(kernel, "kind", None),
                               writer=B200_WRITER)
    if seg.guard is not None or len(seg.segments) != 2 or len(seg.loops) != 1:
        return None
    loop = seg.loops[0]
    if loop.exit == "false" or loop.bounds is not None or (loop.start, loop.by) != (0, 1) or loop.trips < 2:
        return None
    pre, post = body_text(seg.segments[0]), body_text(seg.segments[1])
    step = body_text(loop.step)
    declared = []
    for line in pre.splitlines():
        m = _DECL.match(line)
        if m:
            declared.append(m.group(1))
    used = set(_WORD.findall(step)) | set(_WORD.findall(post))
    lives = []
    for name in declared:
        if name not in used:
            continue
        t = seg.types.get(name)
        if t is None:
            return None
        lives.append((f"hk_l{len(lives)}", body_text(carry_type(t)), name))
    carries = [(f"hk_c{j}", body_text(carry_type(t)), cname, body_text(init), nxt)
               for j, (cname, t, init, nxt) in enumerate(loop.carries)]
    span = 32 * SPAN_ROWS
    p12, p16 = " " * 12, " " * 16

    def bind(indent: str) -> list:
        return ([f"{indent}const {ct} {cname} = {reg};" for reg, ct, cname, _i, _n in carries]
                + [f"{indent}const {lt} {lname} = {reg};" for reg, lt, lname in lives]
                + [f"{indent}(void){cname};" for _r, _c, cname, _i, _n in carries]
                + [f"{indent}(void){lname};" for _r, _l, lname in lives])

    lines = [
        f"    // lane refill: warp w owns the spans of {span} samples at (w + k W) * {span}; a lane takes",
        "    // the next sample of its warp's span the trip its own sample leaves the loop",
        *[f"    {ct} {reg}{{}};" for reg, ct, _c, _i, _n in carries],
        *[f"    {lt} {reg}{{}};" for reg, lt, _l in lives],
        "    const long long hk_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;",
        "    const unsigned hk_lane = threadIdx.x & 31u;",
        f"    long long hk_next = hk::warp_first() * {span}LL;   // the warp's next unclaimed sample",
        f"    long long hk_end = hk_next + {span}LL;             // the end of its current span",
        "    long long hk_flat = 0;",
        "    bool hk_has = false;",
        "    int hk_trip = 0;",
        "    (void)nSamples;",
        "    while (true) {",
        "        const bool hk_needy = !hk_has;",
        "        const unsigned hk_need = __ballot_sync(0xffffffffu, hk_needy);",
        "        if (hk_need != 0u) {",
        "            if (hk_next >= hk_end) {",
        f"                hk_next = hk_end + (hk_warps - 1) * {span}LL;",
        f"                hk_end = hk_next + {span}LL;",
        "            }",
        "            const long long hk_stop = hk_end < count ? hk_end : count;",
        "            const long long hk_avail = hk_stop > hk_next ? hk_stop - hk_next : 0;",
        "            const long long hk_rank = __popc(hk_need & ((1u << hk_lane) - 1u));",
        "            if (hk_needy && hk_rank < hk_avail) {",
        f"{p16}hk_flat = hk_next + hk_rank;",
        f"{p16}const long long hawk_i = base + hk_flat;",
        f"{p16}const hk::SampleIndex i{{hawk_i}};",
        f"{p16}(void)hawk_i;",
        pre.rstrip("\n"),
        *[f"{p16}{reg} = {init};" for reg, _ct, _c, init, _n in carries],
        *[f"{p16}{reg} = {lname};" for reg, _lt, lname in lives],
        f"{p16}hk_trip = 0;",
        f"{p16}hk_has = true;",
        "            }",
        "            const long long hk_took = __popc(hk_need);",
        "            hk_next += hk_took < hk_avail ? hk_took : hk_avail;",
        "        }",
        "        if (!__any_sync(0xffffffffu, hk_has)) {",
        f"            if (hk_next >= count || (hk_next >= hk_end && hk_end + (hk_warps - 1) * {span}LL >= count)) break;",
        "            continue;",
        "        }",
        "        if (hk_has) {",
        f"{p12}const long long hawk_i = base + hk_flat;",
        f"{p12}const hk::SampleIndex i{{hawk_i}};",
        f"{p12}(void)hawk_i;",
        f"{p12}const Int {loop.index} = static_cast<Int>(hk_trip);",
        f"{p12}(void){loop.index};",
        *bind(p12),
        step.rstrip("\n"),
        *[f"{p12}{reg} = {nxt};" for reg, _ct, _c, _i, nxt in carries],
        f"{p12}++hk_trip;",
        f"{p12}if ({loop.exit} || hk_trip >= {loop.trips}) {{",
        *bind(p16),
        post.rstrip("\n"),
        f"{p16}hk_has = false;",
        f"{p12}}}",
        "        }",
        "    }",
    ]
    return "\n".join(lines)
