"""Mirror of the reference's CatalogBackend (directml-model-catalog/.../catalog/CatalogBackend.java) with
the CUDA constant this backend adds: the backends a model family can declare, and their lower-case tokens
(CatalogBackend.token()).  CUDA is the B200 path of this library; like the reference's strict hosts it has
no CPU fallback."""
from __future__ import annotations

import enum


class CatalogBackend(enum.Enum):
    CPU = "CPU"
    DIRECTML = "DIRECTML"
    WARP = "WARP"
    AUTO = "AUTO"
    CUDA = "CUDA"

    def token(self) -> str:
        return self.name.lower()

    @classmethod
    def parse(cls, token: str) -> "CatalogBackend":
        """The backend of a token ("cuda", "CUDA", ...); unknown tokens raise ValueError."""
        try:
            return cls[token.strip().upper()]
        except KeyError:
            raise ValueError(f"unknown backend {token!r}; expected one of "
                             f"{', '.join(b.token() for b in cls)}") from None
