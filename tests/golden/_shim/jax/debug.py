def print(*args, **kwargs):  # noqa: A001 - mirrors jax.debug.print
    return None
