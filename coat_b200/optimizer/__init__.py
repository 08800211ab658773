from .fp8_adamw import CoatAdamW, Coatadamw  # noqa: F401
