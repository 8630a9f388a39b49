"""Model assembly."""

from .bitnet import BitNetModel, create_model  # noqa: F401
from .transformer import TransformerBlock  # noqa: F401
