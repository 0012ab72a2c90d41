"""Emmy dtypes as PTX sees them: register and memory types, register classes, sizes, literals."""

from __future__ import annotations

import struct

# Emmy dtype -> (PTX type of its registers and arithmetic, PTX type it loads and stores as).
# 16-bit floats travel as raw .b16 (ld/st take no .f16/.bf16 type); u8 lives in a 16-bit register.
_TYPES = {
    "f32": ("f32", "f32"), "f64": ("f64", "f64"), "f16": ("f16", "b16"), "bf16": ("bf16", "b16"),
    "u8": ("u16", "u8"), "i16": ("s16", "s16"), "u16": ("u16", "u16"), "i32": ("s32", "s32"),
    "u32": ("u32", "u32"), "i64": ("s64", "s64"), "u64": ("u64", "u64"), "bool": ("pred", "pred"),
}
FLOAT_TYPES = frozenset({"f32", "f64", "f16", "bf16"})

# PTX type -> (register name prefix, .reg declaration type). Types of one width share a class,
# which ptxas accepts (a shfl.b32 can take an .f32 register).
_CLASS = {"pred": ("%p", "pred"), "f32": ("%f", "f32"), "f64": ("%fd", "f64")}
_CLASS |= dict.fromkeys(("b16", "s16", "u16", "u8", "f16", "bf16"), ("%h", "b16"))
_CLASS |= dict.fromkeys(("b32", "s32", "u32"), ("%r", "b32"))
_CLASS |= dict.fromkeys(("b64", "s64", "u64"), ("%rd", "b64"))
REG_PREFIXES = ("%p", "%h", "%r", "%rd", "%f", "%fd")

_SIZE = {"pred": 1, "u8": 1, "b8": 1}
_SIZE |= dict.fromkeys(("b16", "s16", "u16", "f16", "bf16"), 2)
_SIZE |= dict.fromkeys(("b32", "s32", "u32", "f32"), 4)
_SIZE |= dict.fromkeys(("b64", "s64", "u64", "f64"), 8)

# Emmy's C-style names for shared buffers (Smem.dtype) -> Emmy dtype.
C_NAMES = {"float": "f32", "double": "f64", "half": "f16", "__half": "f16",
           "__nv_bfloat16": "bf16", "bfloat16": "bf16", "int": "i32", "int32_t": "i32",
           "unsigned": "u32", "unsigned int": "u32", "uint32_t": "u32", "long long": "i64",
           "int64_t": "i64", "unsigned long long": "u64", "uint64_t": "u64"}


def reg_type(dtype: str) -> str:
    """The PTX register type of an Emmy dtype."""
    if dtype not in _TYPES:
        raise NotImplementedError(f"dtype {dtype}")
    return _TYPES[dtype][0]


def mem_type(dtype: str) -> str:
    """The PTX type an Emmy dtype is loaded and stored as."""
    if dtype not in _TYPES:
        raise NotImplementedError(f"dtype {dtype}")
    return _TYPES[dtype][1]


def reg_class(typ: str) -> tuple[str, str]:
    return _CLASS[typ]


def size(typ: str) -> int:
    """Bytes of a PTX type, or of an Emmy dtype's memory type."""
    if typ in _SIZE:
        return _SIZE[typ]
    return _SIZE[mem_type(typ)]


def move_type(typ: str) -> str:
    """The type suffix mov/selp take for a register of PTX type ``typ``."""
    return "b16" if typ in ("f16", "bf16") else typ


def is_float(dtype: str) -> bool:
    return reg_type(dtype) in FLOAT_TYPES


def is_int(dtype: str) -> bool:
    """An integer Emmy dtype (bool is not one)."""
    return dtype != "bool" and reg_type(dtype) not in FLOAT_TYPES


def smem_dtype(name: str) -> str:
    """An Smem's dtype as an Emmy dtype name."""
    return C_NAMES.get(name, name)


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def bf16_bits(x: float) -> int:
    """Round an f32 value to bf16, nearest even, as raw bits."""
    b = f32_bits(x)
    if (b & 0x7F800000) == 0x7F800000 and b & 0x7FFFFF:
        return 0x7FC0  # a NaN stays a NaN
    return (b + 0x7FFF + ((b >> 16) & 1)) >> 16


def literal(value: float, typ: str) -> str:
    """``value`` as an exact PTX immediate of type ``typ``: hex for floats, so bits survive."""
    if typ == "f32":
        return f"0f{f32_bits(value):08X}"
    if typ == "f64":
        return f"0d{struct.unpack('<Q', struct.pack('<d', value))[0]:016X}"
    if typ == "f16":
        try:
            return f"0x{struct.unpack('<H', struct.pack('<e', value))[0]:04X}"
        except OverflowError:
            return "0xFC00" if value < 0 else "0x7C00"
    if typ == "bf16":
        return f"0x{bf16_bits(value):04X}"
    if typ == "pred":
        return "1" if value else "0"
    if not float(value).is_integer():
        raise ValueError(f"{typ} literal {value!r} is not an integer")
    return str(int(value))
