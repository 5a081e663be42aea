"""Error types of the backend, mirroring catnn's CatError
(crates/catnn-core/src/error.rs:9-54): a status code from the C ABI maps to
the variant the reference returns for the same condition."""


class CatError(Exception):
    """Base of all backend errors (CatError in the reference)."""

    code = -1


class ShapeMismatch(CatError):
    code = 1


class DTypeMismatch(CatError):
    code = 2


class UnknownPort(CatError):
    code = 3


class UnknownComponent(CatError):
    """Raised on the host only (no C-ABI status maps to it)."""
    code = 11


class Wiring(CatError):
    code = 4


class Unlawful(CatError):
    code = 5


class CudaError(CatError):
    code = 6


class InvalidArgument(CatError):
    code = 7


class DeviceTimeout(CatError):
    code = 8


class Unsupported(CatError):
    code = 9


class CommError(CatError):
    code = 10


class Fibration(CatError):
    """An activation that cannot be rebuilt on this device (raised on the host
    only, as coord.rs:443-458 does)."""
    code = 12


_BY_CODE = {cls.code: cls for cls in (ShapeMismatch, DTypeMismatch, UnknownPort, Wiring, Unlawful, CudaError,
                                      InvalidArgument, DeviceTimeout, Unsupported, CommError)}


def raise_for(code, msg):
    raise _BY_CODE.get(code, CatError)(msg)
