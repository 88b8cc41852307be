"""mlx.utils stand-in (numpy).  Fixture generation only."""


def tree_flatten(tree, prefix=""):
    """Flatten nested dicts / lists into [(dotted_name, leaf)] (MLX's documented order)."""
    out = []
    if isinstance(tree, dict):
        for k, v in tree.items():
            out += tree_flatten(v, f"{prefix}{k}.")
    elif isinstance(tree, (list, tuple)):
        for i, v in enumerate(tree):
            out += tree_flatten(v, f"{prefix}{i}.")
    else:
        out.append((prefix[:-1], tree))
    return out


def tree_map(fn, tree):
    if isinstance(tree, dict):
        return {k: tree_map(fn, v) for k, v in tree.items()}
    if isinstance(tree, (list, tuple)):
        return type(tree)(tree_map(fn, v) for v in tree)
    return fn(tree)
