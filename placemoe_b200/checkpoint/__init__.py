from .checkpointer import export_hf, load_checkpoint, load_hf_weights, placement_digest, save_checkpoint

__all__ = ["export_hf", "load_checkpoint", "load_hf_weights", "placement_digest", "save_checkpoint"]
