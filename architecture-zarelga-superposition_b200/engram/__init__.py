"""Drop-in package with the reference's module path (GramReaperSparse); modules it
does not provide are looked up in the same-named package further along sys.path."""
from pkgutil import extend_path

__path__ = extend_path(__path__, __name__)

from .GramReaperSparse import GramReaperSparse

__all__ = ["GramReaperSparse"]
