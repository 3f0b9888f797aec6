"""Data-parallel training support: fp32-master AdamW (optim) and resumable
training checkpoints (checkpoint), the counterparts of the reference's
training/optim.py and training/checkpoint.py."""
