"""Host<->device byte counters for end-to-end accounting (inputs copied from
pinned host memory to the GPU, results read back)."""

H2D = 0
D2H = 0


def h2d(nbytes: int) -> None:
    global H2D
    H2D += int(nbytes)


def d2h(nbytes: int) -> None:
    global D2H
    D2H += int(nbytes)


def snapshot() -> tuple[int, int]:
    return H2D, D2H
