"""Stop strings over decoded text, shared by the offline text API and the
HTTP server: where one begins, how much of a stream's tail may still become
one, and the shortest token prefix whose text holds one."""


def find_stop(text: str, stops) -> int:
    """Index of the earliest stop string in ``text``, or -1."""
    hits = [i for i in (text.find(x) for x in stops) if i >= 0]
    return min(hits) if hits else -1


def held_back(text: str, stops) -> int:
    """Characters at the end of ``text`` that could begin a stop string (a
    stream holds them until the next tokens decide)."""
    hold = 0
    for x in stops:
        for k in range(min(len(x) - 1, len(text)), hold, -1):
            if text.endswith(x[:k]):
                hold = k
                break
    return hold


def stop_prefix(tokens, stops, detok):
    """Length of the shortest token prefix whose text contains a stop string
    (None if the whole output holds none)."""
    if find_stop(detok(tokens), stops) < 0:
        return None
    k = len(tokens)
    while k > 1 and find_stop(detok(tokens[:k - 1]), stops) >= 0:
        k -= 1
    return k


def tail_hit(tokens, stops, detok) -> bool:
    """Whether the newest tokens complete a stop string: decodes a tail window
    long enough for the longest one, not the whole output."""
    win = max(16, 4 * max(len(x) for x in stops))
    return find_stop(detok(tokens[-win:]), stops) >= 0
