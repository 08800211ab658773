"""QuantizationConfig: the knob set the reference passes around as `qargs`
(coat/utils/_fp8_quantization_config.py:6-80).  Field names, types, defaults, their order (it is the positional
order of the constructor) and the tolerance for unknown keyword arguments follow the reference, so that configs,
HfArgumentParser command lines and `coat_fp8_args` dictionaries written for it keep working.  One quirk is kept:
the dataclass default of `pad_to_multiple_of` is 8 while the constructor's default is 0.

The class is generated from the table below instead of being spelled out three times."""
import dataclasses

# name, type, dataclass default, constructor default
_FIELDS = [
    # activations and linears
    ("quantize_model", str, "true", "true"),
    ("symm", bool, True, True),
    ("epsilon", float, 1e-10, 1e-10),
    ("fabit", str, "E4M3", "E4M3"),
    ("fwbit", str, "E4M3", "E4M3"),
    ("fobit", str, "E4M3", "E4M3"),
    ("babit", str, "E5M2", "E5M2"),
    ("bwbit", str, "E5M2", "E5M2"),
    ("bobit", str, "E5M2", "E5M2"),
    ("group_size", int, 16, 16),
    ("pad_to_multiple_of", int, 8, 0),
    ("weight_memory_efficient", bool, True, True),
    # optimizer states
    ("first_order_expansion", str, "true", "true"),
    ("second_order_expansion", str, "true", "true"),
    ("first_order_bit", str, "E4M3", "E4M3"),
    ("second_order_bit", str, "E4M3", "E4M3"),
    ("qgroup_size", int, 128, 128),
    ("expand_min", int, 16, 16),
    # legacy
    ("row_blocksize", int, -1, -1),
    ("col_blocksize", int, -1, -1),
]


def _init(self, *args, **kwargs):
    if len(args) > len(_FIELDS):
        raise TypeError(f"QuantizationConfig takes at most {len(_FIELDS)} positional arguments")
    values = {name: ctor_default for name, _, _, ctor_default in _FIELDS}
    for (name, _, _, _), value in zip(_FIELDS, args):
        values[name] = value
    for name in values:
        if name in kwargs:
            values[name] = kwargs[name]   # keys that are not fields are ignored, as in the reference
    for name, value in values.items():
        setattr(self, name, value)


QuantizationConfig = dataclasses.make_dataclass(
    "QuantizationConfig",
    [(name, typ, dataclasses.field(default=default)) for name, typ, default, _ in _FIELDS],
    namespace={"__init__": _init, "__module__": __name__, "__doc__": __doc__},
    init=False,
)
