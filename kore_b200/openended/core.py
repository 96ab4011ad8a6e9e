"""Single import point of the open-ended curriculum (task space, archive,
proposer, controller, loop)."""
from .archive import ArchiveEntry, DescriptorStats, TaskArchive  # noqa: F401
from .coevolve import coevolve, frontier_report  # noqa: F401
from .controller import CoevolutionController, CurriculumController  # noqa: F401
from .proposer import Proposer  # noqa: F401
from .task_space import TaskDescriptor, TaskSpace  # noqa: F401
