"""TEST INFRASTRUCTURE ONLY: a stand-in for the third-party ``dahuffman`` package.

The reference codec imports ``from dahuffman import HuffmanCodec``
(dfloat/utils.py:7) and uses exactly four things from it:
``HuffmanCodec.from_frequencies`` (utils.py:240,259), ``get_code_table()``
(utils.py:241,260), ``codec._table[symbol]`` (utils.py:408) and
``codec._eof`` (utils.py:447).  ``dahuffman`` is unpinned in the reference's
requirements.txt:34 and is not installed in this image, so this module
restates the algorithm dahuffman publishes for ``from_frequencies``: a
textbook Huffman (1952) merge over a binary heap of
``(frequency, [(symbol, (bit_count, code_value)), ...])`` nodes, where an EOF
pseudo-symbol of frequency 1 is added, the two least frequent nodes are
popped, the first popped gets a 0 prefix bit and the second a 1 prefix bit,
and the merged node is pushed back.  Ties between equal frequencies are broken
by comparing the leaf lists, with the EOF symbol ordering before every real
symbol.

Only ``tests/golden/make_fixtures.py`` puts this directory on ``sys.path`` so
that the reference's ``dfloat/utils.py`` imports in this container.  The code
tables it produces are recorded in the fixtures, so no test depends on it.
Decode parity does not depend on the exact table either: the LUTs that carry
the code are part of every stream.
"""

from heapq import heapify, heappop, heappush

__all__ = ["HuffmanCodec"]


class _EndOfFile:
    """EOF pseudo-symbol; orders before every real symbol on ties."""

    def __repr__(self):
        return "_EOF"

    def __lt__(self, other):
        return not isinstance(other, _EndOfFile)

    def __gt__(self, other):
        return False

    def __eq__(self, other):
        return isinstance(other, _EndOfFile)

    def __hash__(self):
        return hash(_EndOfFile)


_EOF = _EndOfFile()


class HuffmanCodec:
    def __init__(self, table, eof=_EOF):
        self._table = table
        self._eof = eof

    @classmethod
    def from_frequencies(cls, frequencies, concat=None, eof=_EOF):
        heap = [(f, [(s, (0, 0))]) for s, f in frequencies.items()]
        if eof not in frequencies:
            heap.append((1, [(eof, (0, 0))]))
        heapify(heap)
        while len(heap) > 1:
            lo = heappop(heap)
            hi = heappop(heap)
            merged = (
                lo[0] + hi[0],
                [(s, (n + 1, v)) for (s, (n, v)) in lo[1]]
                + [(s, (n + 1, (1 << n) + v)) for (s, (n, v)) in hi[1]],
            )
            heappush(heap, merged)
        return cls(dict(heap[0][1]), eof=eof)

    def get_code_table(self):
        return self._table
