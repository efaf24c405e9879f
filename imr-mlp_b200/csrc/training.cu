// training.cu -- loss and coefficient gradient of a structure batch.
#include "context.hpp"

namespace mtpb {

int loss_grad_compute(mtpb_context *c, const mtpb_labels *labels, const mtpb_loss_weights *w,
                      int norm_count, int memory, double *loss, double *metrics, double *grad)
{
    (void)labels;
    (void)w;
    (void)norm_count;
    (void)memory;
    (void)loss;
    (void)metrics;
    (void)grad;
    if (!c)
        return fail(MTPB_ERR_ARGUMENT, "ctx is NULL");
    return fail(MTPB_ERR_UNSUPPORTED, "mtpb_loss_grad is not available in this build");
}

} // namespace mtpb
