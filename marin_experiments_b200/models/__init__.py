from .grug import Transformer, apply_qb_betas, combine_losses, default_loss_weight  # noqa: F401
