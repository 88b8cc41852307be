"""numpy-backed stand-in for the parts of MLX that rwkv_mlx's model.py, moe.py and
kernels/wkv7_metal.py use (fixture generation only; see tests/golden/make_golden.py).

MLX (`mlx>=0.22.0`, unpinned in the reference's pyproject.toml) is not installable
here.  Each function restates MLX's documented behaviour on numpy arrays; arrays are
plain numpy arrays (float32 / float16 / uint32), evaluated eagerly.
"""
