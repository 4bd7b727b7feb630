"""Rounding modes with the stable integer codes the C ABI uses (``tricast/rounding.py:14-40``)."""

from __future__ import annotations

from enum import Enum


class Rounding(str, Enum):
    RNE = "rne"
    RNA = "rna"
    RTZ = "rtz"
    RUP = "rup"
    RDN = "rdn"
    SR = "sr"

    @classmethod
    def parse(cls, value) -> "Rounding":
        if isinstance(value, Rounding):
            return value
        key = getattr(value, "value", value)
        key = str(key).strip().lower()
        key = {"even": "rne", "trunc": "rtz", "truncate": "rtz", "stochastic": "sr"}.get(key, key)
        try:
            return cls(key)
        except ValueError:
            raise ValueError(f"unknown rounding {value!r}; use one of {[r.value for r in cls]}") from None

    @property
    def code(self) -> int:
        return CODES[self.value]


CODES = {"rne": 0, "rna": 1, "rtz": 2, "rup": 3, "rdn": 4, "sr": 5}


def rounding_code(value) -> int:
    """Integer code of a rounding given as our enum, TriCast's enum or a string."""
    return CODES[Rounding.parse(value).value]
