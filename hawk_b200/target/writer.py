"""The b200 writer: how the body spells each construct for the sm_100a device library.

The reference's Writer protocol (hawk/emit/writer.py:29-191) is answered by the
reference's aether spelling (``AetherWriter``, hawk/emit/writer_aether.py:124),
with two changes:

* the library namespace the text names is this build's device library
  (``hk::``, hawk_b200/csrc/include/hk) -- its types and functions keep the
  names that spelling uses (``Item``, ``linalg::cholesky``, ``math::sin``, ...),
  because the renderer's text is written in them;
* no site is spelled as a rolled runtime twin (``rolled_forms = False`` and a
  plain own-column store): every small vector or matrix stays an unrolled,
  register-resident value, which is what a one-sample-per-thread sm_100a lane
  wants, and the device library needs no runtime-index twins.

This module imports the reference's front end (to subclass its writer).
"""

from __future__ import annotations

from hawk.emit.writer_aether import AetherWriter


class B200Writer(AetherWriter):
    """The aether spelling, rendered for the hk device library."""

    id = "b200"
    rolled_forms = False

    def _team_read(self, r, node, plane: str) -> str:
        """A vector or matrix a team stage left in the lane's slice of its
        scratch plane: a view of the slice (``hk::Slice``), read element by
        element where it is used and copied by the rolled store, instead of a
        fresh value of every element (hawk/emit/writer_aether.py:342-352),
        which at the team form's sizes (hundreds to thousands of elements)
        would live in local memory."""
        from math import prod

        from hawk.emit.spelling import element_spelling

        shape = node.ttype.shape
        if not shape:
            return super()._team_read(r, node, plane)
        size = prod(shape)
        name = f"hawk_la{r.hoists}"
        r.hoists += 1
        extents = ", ".join(str(int(e)) for e in shape)
        base = f"static_cast<std::size_t>({r._ref(node.index)}) * {size}"
        r._emit(f"const hk::Slice<{element_spelling(node.ttype.dtype)}, {extents}> {name}{{{plane}.data() + {base}}};")
        r.proxies.add(name)
        return name

    def store(self, r, sink, target: str, value: str) -> None:
        """The own column: one store of the whole value (a register Item or
        scalar), or nothing when a library call already wrote the plane; a
        value that lives in a plane (a team stage's result) is copied by the
        rolled store."""
        if value == f"{target}[i]":
            return
        if value in r.proxies:
            r._emit(f"hk::rt::store({target}[i], {value});")
            return
        r._emit(f"{target}[i] = {value};")


#: The one b200 writer instance (stateless, like the reference's AETHER).
B200_WRITER = B200Writer()


def body_text(text: str) -> str:
    """The rendered body in the device library's namespace."""
    return text.replace("aether::", "hk::")
