"""``has_triton`` is False so the reference registers no Triton ops on import."""


def has_triton() -> bool:
    return False
