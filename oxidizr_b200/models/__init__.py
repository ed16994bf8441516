"""Model zoo: GQA / MLA / MoE / Mamba1 / Mamba2 / Mamba3 blocks and the LM."""
from .model import LitGPT, build_model, make_block  # noqa: F401
