from .GramReaperSparse import GramReaperSparse

__all__ = ["GramReaperSparse"]
