"""mlx.optimizers stand-in: present so that rwkv_mlx/train.py imports (its loss
functions are used for fixtures; no optimizer runs).  Fixture generation only."""
