"""Drop-in package with the reference's module path.  Modules this package does
not provide (for example the reference's own helpers that are not part of the
training step) are looked up in the same-named package further along sys.path,
so an import root placed in front of a reference checkout shadows only what it
replaces."""
from pkgutil import extend_path

__path__ = extend_path(__path__, __name__)
