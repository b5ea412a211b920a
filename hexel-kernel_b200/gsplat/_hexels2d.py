"""2D image-hexel entry points of ``gsplat.csrc`` (filled in below)."""


def exports() -> dict:
    return {}
