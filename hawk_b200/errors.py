"""The one refusal type of the b200 path.

Every refusal names what failed, as the reference's ``HawkError``
(hawk/ir/nodes.py:24) does: a bind that does not match the artifact, a kernel
construct the target does not build, a C-ABI call that returned an error
status (its message is the library's thread-local error text).
"""


class HawkError(Exception):
    """A refusal of the b200 path, naming every failing argument."""
